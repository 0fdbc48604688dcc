"""GPU parity of mv_small_linear (fastlinear.small_linear drop-in) against the reference kernel's golden vectors
and the oracle at the reference's shapes (shared-expert gate_up 2048 -> 5632, down 2816 -> 2048)."""
import pytest
import torch

import fastlinear
from conftest import golden
from oracle import moe_oracle as O

pytestmark = pytest.mark.gpu


def test_small_linear_golden(cuda):
    d = golden("small_linear")
    g = {k: (v.to(cuda) if torch.is_tensor(v) else v) for k, v in d.items()}
    cases = {
        "y_plain": dict(),
        "y_bias_gelu_res": dict(b=g["b"], act=1, residual=g["r"]),
        "y_silu": dict(act=2),
        "y_norm_bias": dict(b=g["b"], norm=(g["gamma"], d["eps"])),
        "y_norm_gelu_res": dict(b=g["b"], act=1, residual=g["r"], norm=(g["gamma"], d["eps"])),
    }
    for name, kw in cases.items():
        y = fastlinear.small_linear(g["x"], g["w"], **kw).float().cpu()
        ref = d[name].float()
        assert (y - ref).abs().max().item() <= 2e-2, name  # the reference kernel's own output (bf16)


@pytest.mark.parametrize("M", [1, 3, 16])
@pytest.mark.parametrize("N,K", [(5632, 2048), (2048, 2816), (896, 896)])
def test_small_linear_reference_shapes(cuda, M, N, K):
    gen = torch.Generator().manual_seed(M * 7 + N)
    x = torch.randn(M, K, generator=gen).to(torch.bfloat16)
    w = (torch.randn(N, K, generator=gen) * 0.02).to(torch.bfloat16)
    b = (torch.randn(N, generator=gen) * 0.1).to(torch.bfloat16)
    r = torch.randn(M, N, generator=gen).to(torch.bfloat16)
    gam = (1 + 0.1 * torch.randn(K, generator=gen)).to(torch.bfloat16)
    for kw in (dict(), dict(b=b, act=2), dict(b=b, act=1, residual=r, norm=(gam, 1e-6))):
        ref = O.small_linear(x, w, **kw).to(torch.bfloat16).float()
        kwg = {k: (tuple(t.cuda() if torch.is_tensor(t) else t for t in v) if isinstance(v, tuple) else
                   (v.cuda() if torch.is_tensor(v) else v)) for k, v in kw.items()}
        y = fastlinear.small_linear(x.cuda(), w.cuda(), **kwg).float().cpu()
        d = (y - ref).abs()
        assert d.max().item() <= 2e-2
        assert (d.sum() / ref.abs().sum()).item() <= 1e-2


def test_small_linear_shapes_and_out(cuda):
    x = torch.randn(2, 3, 256, device=cuda).to(torch.bfloat16)
    w = (torch.randn(64, 256, device=cuda) * 0.05).to(torch.bfloat16)
    out = torch.empty(6, 64, device=cuda, dtype=torch.bfloat16)
    y = fastlinear.small_linear(x, w, out=out)
    assert y.shape == (2, 3, 64) and y.data_ptr() == out.data_ptr()
    assert fastlinear.save_cache() is None
    t = fastlinear._graph_time(lambda: fastlinear.small_linear(x, w, out=out), reps=2, inner=2)
    assert t > 0
    x17 = torch.randn(17, 256, device=cuda).to(torch.bfloat16)  # > 16 rows: the reference's torch path
    assert fastlinear.small_linear(x17, w).shape == (17, 64)
