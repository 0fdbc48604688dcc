"""The oracle against golden vectors produced by the reference's own kernels (tests/golden/make_golden.py).

In rounding="reference" mode the oracle must reproduce the reference kernels bit for bit: same rounding
points, same selection order, same integer results."""
import numpy as np
import torch

from conftest import golden
from oracle import moe_oracle as O


def test_rms_norm_matches_reference_kernel():
    d = golden("rms_norm")
    y = O.rms_norm(d["x"], d["w"], d["eps"])
    assert y.dtype == d["y"].dtype
    assert torch.equal(y, d["y"])


def test_route_sigmoid_group_matches_reference_kernel():
    d = golden("moe_route")
    ids, wts, logits = O.route_sigmoid_group(d["x"], d["w32"], d["bias"], d["n_group"], d["topk_group"],
                                             d["top_k"], d["scale"])
    assert torch.equal(ids, d["ids"])
    # tied experts 5, 9, 40 (identical router rows) come out lowest id first
    assert ids[5, :3].tolist() == [5, 9, 40]
    assert torch.allclose(wts, d["wts"], rtol=0, atol=2e-7)
    assert torch.allclose(logits, d["logits"], rtol=2e-5, atol=1e-6)
    assert (ids[:, -1] == d["w32"].shape[0]).all() and (wts[:, -1] == 1.0).all()


def test_quantize_rows_int8_bit_exact():
    d = golden("quantize_rows_int8")
    q, s = O.quantize_rows_int8(d["w"])
    assert torch.equal(q, d["q"]) and torch.equal(s, d["scale"])


def test_align_blocks_bit_exact():
    d = golden("align_blocks")
    si, be, nb = O.align_blocks(d["flat"].numpy(), d["E1"], d["BM"])
    assert nb == d["nb"]
    assert np.array_equal(si, d["sorted_ids"].numpy()) and np.array_equal(be, d["bexp"].numpy())


def _experts(d, int8, rounding):
    kw = dict(s_gu=d["s_gu"], s_d=d["s_d"]) if int8 else {}
    wg = d["q_gu"] if int8 else d["w_gu"]
    wd = d["q_d"] if int8 else d["w_d"]
    return O.moe_experts(d["x"], wg, wd, d["ids"], d["wts"], rounding=rounding, **kw)


def test_moe_decode_matches_reference_kernel():
    d = golden("moe_decode")
    for int8, key in ((False, "y"), (True, "y_int8")):
        y = _experts(d, int8, "reference").to(torch.bfloat16)
        assert torch.equal(y, d[key]), key
        # and the fp32 oracle is within bf16 rounding of it
        y32 = _experts(d, int8, "fp32")
        assert (y32 - d[key].float()).abs().max() < 2e-3


def test_moe_prefill_matches_reference_kernel():
    d = golden("moe_prefill")
    for int8, key in ((False, "y"), (True, "y_int8")):
        y = _experts(d, int8, "reference").to(torch.bfloat16)
        assert torch.equal(y, d[key]), key
        y32 = _experts(d, int8, "fp32")
        assert (y32 - d[key].float()).abs().max() < 1e-2


def test_small_linear_matches_reference_kernel():
    d = golden("small_linear")
    cases = {"plain": {}, "bias_gelu_res": dict(b=d["b"], act=1, residual=d["r"]), "silu": dict(act=2),
             "norm_bias": dict(b=d["b"], norm=(d["gamma"], d["eps"])),
             "norm_gelu_res": dict(b=d["b"], act=1, residual=d["r"], norm=(d["gamma"], d["eps"]))}
    for name, kw in cases.items():
        y = O.small_linear(d["x"], d["w"], **kw).to(torch.bfloat16)
        assert torch.equal(y, d["y_" + name]), name


def test_softmax_router_tie_break_and_renorm():
    H, E = 64, 16
    w = torch.randn(E, H).to(torch.bfloat16)
    w[7] = w[3]
    w[12] = w[3]
    x = (w[3].float() * 5).to(torch.bfloat16)[None]
    ids, wts, _ = O.route_softmax(x, w, top_k=4, shared_ids=(16, 17))
    assert ids[0, :3].tolist() == [3, 7, 12]
    assert ids[0, 4:].tolist() == [16, 17]
    assert abs(wts[0, :4].double().sum().item() - 1.0) < 1e-6
    assert (wts[0, 4:] == 1).all()


def test_shared_expert_split_is_exact_swiglu():
    """A 2I-wide shared SwiGLU expert equals two I-wide slots with weight 1 (the slot split used for
    BASELINE's I_s = 2816 = 2 x 1408)."""
    p = O.make_block_params(seed=3, H=64, I=16, E=4, I_s=32, dtype=torch.float32)
    x = torch.randn(3, 64)
    ids = torch.tensor([[4, 5]] * 3)
    wts = torch.ones(3, 2)
    y = O.moe_experts(x, p["w_gu"], p["w_d"], ids, wts)
    g = torch.cat([p["w_gu"][4, :16], p["w_gu"][5, :16]])
    u = torch.cat([p["w_gu"][4, 16:], p["w_gu"][5, 16:]])
    dn = torch.cat([p["w_d"][4], p["w_d"][5]], 1)
    ref = (torch.nn.functional.silu(x @ g.T) * (x @ u.T)) @ dn.T
    assert torch.allclose(y, ref, atol=1e-5)
