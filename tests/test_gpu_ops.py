"""GPU parity: RMSNorm, router, int8 quantiser / dequantiser against the oracle and the reference goldens.

Bar: bit-exact for integer results (top-k ids, int8 q and scales, dequantised values) and for the RMSNorm,
whose arithmetic is fully specified; fp32 router weights within a few ulp."""
import pytest
import torch

import fused_moe
import fused_ops
from conftest import golden
from oracle import moe_oracle as O

pytestmark = pytest.mark.gpu


def test_rms_norm_golden_and_oracle(cuda):
    d = golden("rms_norm")
    y = fused_ops.rms_norm(d["x"].to(cuda), d["w"].to(cuda), d["eps"])
    assert torch.equal(y.cpu(), d["y"])
    g = torch.Generator().manual_seed(5)
    for rows, n, xd, wd in ((1, 2048, torch.bfloat16, torch.bfloat16), (37, 2048, torch.bfloat16, torch.bfloat16),
                            (5, 1536, torch.bfloat16, torch.float32), (3, 4096, torch.float32, torch.float32),
                            (2, 1000, torch.float16, torch.float16)):
        x = (torch.randn(rows, n, generator=g) * 3).to(xd)
        w = (1 + 0.1 * torch.randn(n, generator=g)).to(wd)
        ref = O.rms_norm(x, w, 1e-6)
        got = fused_ops.rms_norm(x.to(cuda), w.to(cuda), 1e-6).cpu()
        assert got.dtype == ref.dtype
        assert torch.equal(got, ref), (rows, n, xd, wd)


def test_rms_norm_strided_and_empty(cuda):
    x = torch.randn(4, 3, 256, dtype=torch.bfloat16)
    w = torch.ones(256, dtype=torch.bfloat16)
    got = fused_ops.rms_norm(x.to(cuda)[:, 1], w.to(cuda), 1e-5).cpu()
    assert torch.equal(got, O.rms_norm(x[:, 1], w, 1e-5))
    e = fused_ops.rms_norm(torch.empty(0, 256, dtype=torch.bfloat16, device=cuda), w.to(cuda), 1e-5)
    assert e.shape == (0, 256)


def test_quantize_rows_int8_bit_exact(cuda):
    d = golden("quantize_rows_int8")
    q, s = fused_moe.quantize_rows_int8(d["w"].to(cuda))
    assert torch.equal(q.cpu(), d["q"]) and torch.equal(s.cpu(), d["scale"])
    g = torch.Generator().manual_seed(6)
    w = (torch.randn(3, 64, 1408, generator=g) * 0.02).to(torch.bfloat16)
    w[1, 7] = 0
    for sd in (torch.float32, torch.bfloat16):
        q, s = fused_moe.quantize_rows_int8(w.to(cuda), scale_dtype=sd)
        qr, sr = O.quantize_rows_int8(w, sd)
        assert torch.equal(q.cpu(), qr) and torch.equal(s.cpu(), sr), sd
        # the in-kernel dequantisation equals torch's q.float() * s.float(), bit for bit
        deq = fused_moe.dequantize_rows_int8(q, s).cpu()
        assert torch.equal(deq, O.dequant_rows_int8(qr, sr))


def _route_ref_inputs(seed, n, H, E):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(n, H, generator=g).to(torch.bfloat16)
    w = (torch.randn(E, H, generator=g) * 0.02).to(torch.bfloat16)
    return x, w


def test_moe_route_sigmoid_group_golden(cuda):
    d = golden("moe_route")
    E = d["w32"].shape[0]
    K = d["top_k"]
    for t in range(d["x"].shape[0]):
        logits = torch.empty(E, device=cuda)
        ids = torch.empty(K + 1, dtype=torch.long, device=cuda)
        wts = torch.empty(K + 1, device=cuda)
        fused_ops.moe_route(d["x"][t:t + 1].to(cuda), d["w32"].to(cuda), d["bias"].to(cuda), d["n_group"],
                            d["topk_group"], K, d["scale"], logits, ids, wts)
        assert torch.equal(ids.cpu(), d["ids"][t]), t
        assert torch.allclose(wts.cpu(), d["wts"][t], rtol=0, atol=3e-7)
        assert torch.allclose(logits.cpu(), d["logits"][t], rtol=2e-5, atol=1e-6)


@pytest.mark.parametrize("n", [1, 7, 16, 300])
def test_moe_route_sigmoid_group_reference_model_dims(cuda, n):
    # the reference model's router: E=128, H=1536, 8 groups keep 4, top-8, scale 2.5, fp32 w32, bias
    x, w = _route_ref_inputs(21 + n, n, 1536, 128)
    w32 = w.float()
    bias = torch.randn(128, generator=torch.Generator().manual_seed(3)) * 0.05
    ids_r, wts_r, lg_r = O.route_sigmoid_group(x, w32, bias, 8, 4, 8, 2.5)
    ids = torch.empty(n, 9, dtype=torch.long, device=cuda)
    wts = torch.empty(n, 9, device=cuda)
    lg = torch.empty(n, 128, device=cuda)
    fused_ops.moe_route(x.to(cuda), w32.to(cuda), bias.to(cuda), 8, 4, 8, 2.5, lg, ids, wts)
    assert torch.equal(lg.cpu(), lg_r)
    assert torch.equal(ids.cpu(), ids_r)
    assert torch.allclose(wts.cpu(), wts_r, rtol=2e-7, atol=0)


@pytest.mark.parametrize("n", [1, 2, 4, 8, 16, 2043])
def test_route_softmax_baseline_dims(cuda, n):
    x, w = _route_ref_inputs(31 + n, n, 2048, 64)
    bias = O.zipf_bias(64) if n > 16 else None
    ids_r, wts_r, lg_r = O.route_softmax(x, w, bias=bias, top_k=6, shared_ids=(64, 65))
    ids, wts, lg = fused_ops.route_softmax(x.to(cuda), w.to(cuda), 6, bias=None if bias is None else bias.to(cuda),
                                           n_shared=2, shared_id=64)
    assert torch.equal(lg.cpu(), lg_r)
    assert torch.equal(ids.cpu(), ids_r)
    assert torch.allclose(wts.cpu(), wts_r, rtol=2e-7, atol=0)


def test_route_softmax_ties_and_int8_router(cuda):
    H, E = 2048, 64
    x, w = _route_ref_inputs(41, 4, H, E)
    w[17] = w[3]
    w[50] = w[3]
    x[2] = (w[3].float() * 8).to(torch.bfloat16)
    q, s = O.quantize_rows_int8(w, torch.bfloat16)
    for wt, sc in ((w, None), (q, s)):
        ids_r, wts_r, _ = O.route_softmax(x, wt, top_k=6, shared_ids=(64, 65), w_scale=sc)
        ids, wts, _ = fused_ops.route_softmax(x.to(cuda), wt.to(cuda), 6, n_shared=2, shared_id=64,
                                              w_scale=None if sc is None else sc.to(cuda))
        assert torch.equal(ids.cpu(), ids_r)
        assert ids_r[2, :3].tolist() == [3, 17, 50]
        assert torch.allclose(wts.cpu(), wts_r, rtol=2e-7, atol=0)


def test_route_int32_ids_and_errors(cuda):
    x, w = _route_ref_inputs(51, 2, 256, 16)
    ids = torch.empty(2, 3, dtype=torch.int32, device=cuda)
    wts = torch.empty(2, 3, device=cuda)
    fused_ops.moe_route(x.to(cuda), w.to(cuda), None, 1, 1, 2, 1.0, None, ids, wts, mode="softmax")
    ids_r, _, _ = O.route_softmax(x, w, top_k=2, shared_ids=(16,))
    assert torch.equal(ids.cpu().long(), ids_r)
    with pytest.raises(RuntimeError):  # top_k larger than the kept experts
        fused_ops.moe_route(x.to(cuda), w.float().to(cuda), torch.zeros(16, device=cuda), 4, 1, 8, 1.0, None,
                            torch.empty(2, 9, dtype=torch.long, device=cuda), torch.empty(2, 9, device=cuda))
