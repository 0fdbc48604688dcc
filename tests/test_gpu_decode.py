"""GPU parity of the decode MoE kernel (M <= 16): against the reference goldens and the fp32 oracle at
BASELINE dims (H=2048, I=1408, E=64 + 2 shared slots, top-6), bf16 and int8 weights.

Tolerance: bf16 output within max-abs 2e-2 and mean-rel 1e-2 of the fp32 oracle."""
import pytest
import torch

import fused_moe
from conftest import golden
from mingmoe import _lib as L
from mingmoe import moe
from oracle import moe_oracle as O

pytestmark = pytest.mark.gpu

MAX_ABS, MEAN_REL = 2e-2, 1e-2


def close(got, ref, max_abs=MAX_ABS, mean_rel=MEAN_REL):
    got = got.float().cpu()
    ref = ref.float().cpu()
    d = (got - ref).abs()
    mr = (d.sum() / ref.abs().sum().clamp_min(1e-30)).item()
    assert d.max().item() <= max_abs, f"max-abs {d.max().item():.3e}"
    assert mr <= mean_rel, f"mean-rel {mr:.3e}"


def no_device_errors():
    errs = L.all_workspace_errors(clear=True)
    assert not errs, errs


def test_decode_golden_bf16_and_int8(cuda):
    d = golden("moe_decode")
    x, ids, wts = d["x"].to(cuda), d["ids"].to(cuda), d["wts"].to(cuda)
    y = fused_moe.fused_moe_decode(x, d["w_gu"].to(cuda), d["w_d"].to(cuda), ids, wts)
    ref32 = O.moe_experts(d["x"], d["w_gu"], d["w_d"], d["ids"], d["wts"])
    close(y, ref32, max_abs=4e-3)
    close(y, d["y"], max_abs=8e-3)  # the reference kernel rounds intermediates to bf16
    y8 = fused_moe.fused_moe_decode(x, d["q_gu"].to(cuda), d["q_d"].to(cuda), ids, wts, s_gu=d["s_gu"].to(cuda),
                                    s_d=d["s_d"].to(cuda))
    ref8 = O.moe_experts(d["x"], d["q_gu"], d["q_d"], d["ids"], d["wts"], s_gu=d["s_gu"], s_d=d["s_d"])
    close(y8, ref8, max_abs=4e-3)
    close(y8, d["y_int8"], max_abs=8e-3)
    no_device_errors()


@pytest.fixture(scope="module")
def base_params():
    return O.make_block_params(seed=0)


@pytest.fixture(scope="module")
def base_params_gpu(base_params):
    return {k: (v.cuda() if torch.is_tensor(v) else v) for k, v in base_params.items()}


@pytest.mark.parametrize("M", [1, 2, 4, 8, 16])
@pytest.mark.parametrize("seed", [0, 1, 2, 3, 4])
def test_decode_baseline_bf16(cuda, base_params, base_params_gpu, M, seed):
    p, pg = base_params, base_params_gpu
    x = O.make_tokens(M, seed=seed)
    xn = O.rms_norm(x, p["norm_w"], p["eps"])
    ids, wts, _ = O.route_softmax(xn, p["router_w"], top_k=6, shared_ids=p["shared_ids"])
    ref = O.moe_experts(xn, p["w_gu"], p["w_d"], ids, wts)
    got = moe.decode(xn.to(cuda), pg["w_gu"], pg["w_d"], ids.to(cuda), wts.to(cuda))
    close(got, ref)
    # fused RMSNorm prologue + residual epilogue
    got2 = moe.decode(x.to(cuda), pg["w_gu"], pg["w_d"], ids.to(cuda), wts.to(cuda), norm_w=pg["norm_w"],
                      eps=p["eps"], residual=x.to(cuda))
    close(got2, ref + x.float())
    no_device_errors()


@pytest.fixture(scope="module")
def int8_params():
    return O.make_block_params(seed=1, int8=True)


@pytest.mark.parametrize("M", [1, 4, 16])
def test_decode_baseline_int8(cuda, int8_params, M):
    p = int8_params
    pg = {k: (v.cuda() if torch.is_tensor(v) else v) for k, v in p.items()}
    x = O.make_tokens(M, seed=1)
    xn = O.rms_norm(x, p["norm_w"], p["eps"])
    ids, wts, _ = O.route_softmax(xn, p["router_w"], top_k=6, shared_ids=p["shared_ids"], w_scale=p["router_s"])
    ref = O.moe_experts(xn, p["w_gu"], p["w_d"], ids, wts, s_gu=p["s_gu"], s_d=p["s_d"])
    got = moe.decode(xn.to(cuda), pg["w_gu"], pg["w_d"], ids.to(cuda), wts.to(cuda), s_gu=pg["s_gu"], s_d=pg["s_d"])
    close(got, ref)
    no_device_errors()


def test_decode_reference_model_dims_fp32_scales(cuda):
    # ming-voice's thinker: H=1536, I=512, 128 experts + shared slot 128, top-8, fp32 int8 scales
    g = torch.Generator().manual_seed(7)
    E, H, I = 128, 1536, 512
    w_gu = (torch.randn(E + 1, 2 * I, H, generator=g) * 0.02).to(torch.bfloat16)
    w_d = (torch.randn(E + 1, H, I, generator=g) * 0.02).to(torch.bfloat16)
    x = torch.randn(1, H, generator=g).to(torch.bfloat16)
    ids = torch.cat([torch.randperm(E, generator=g)[:8], torch.tensor([E])])
    wts = torch.cat([torch.rand(8, generator=g), torch.ones(1)])
    ref = O.moe_experts(x, w_gu, w_d, ids[None], wts[None])
    got = fused_moe.fused_moe_decode(x.cuda(), w_gu.cuda(), w_d.cuda(), ids.cuda(), wts.cuda())
    close(got, ref)
    q_gu, s_gu = O.quantize_rows_int8(w_gu)
    q_d, s_d = O.quantize_rows_int8(w_d)
    ref8 = O.moe_experts(x, q_gu, q_d, ids[None], wts[None], s_gu=s_gu, s_d=s_d)
    got8 = fused_moe.fused_moe_decode(x.cuda(), q_gu.cuda(), q_d.cuda(), ids.cuda(), wts.cuda(), s_gu=s_gu.cuda(),
                                      s_d=s_d.cuda())
    close(got8, ref8)
    no_device_errors()


def test_decode_edge_cases(cuda, base_params, base_params_gpu):
    p, pg = base_params, base_params_gpu
    x = O.make_tokens(3, seed=9)
    # duplicate expert in one token's list, int32 ids, same expert shared by all tokens
    ids = torch.tensor([[5, 5, 64, 65], [5, 7, 64, 65], [63, 0, 64, 65]], dtype=torch.int32)
    wts = torch.tensor([[0.25, 0.5, 1, 1], [0.3, 0.7, 1, 1], [0.9, 0.1, 1, 1]])
    ref = O.moe_experts(x, p["w_gu"], p["w_d"], ids, wts)
    got = moe.decode(x.to(cuda), pg["w_gu"], pg["w_d"], ids.to(cuda), wts.to(cuda))
    close(got, ref)
    no_device_errors()
    # an out-of-range id is skipped and flagged, never read
    bad = ids.clone()
    bad[1, 1] = 1000
    ref_bad = O.moe_experts(x, p["w_gu"], p["w_d"], torch.where(bad == 1000, 0, bad),
                            torch.where(bad == 1000, torch.zeros_like(wts), wts))
    got = moe.decode(x.to(cuda), pg["w_gu"], pg["w_d"], bad.to(cuda), wts.to(cuda))
    close(got, ref_bad)
    errs = L.all_workspace_errors(clear=True)
    assert any(c == 2 for c, _ in errs.values())
    # repeated calls reuse the self-cleaning workspace
    for _ in range(3):
        got = moe.decode(x.to(cuda), pg["w_gu"], pg["w_d"], ids.to(cuda), wts.to(cuda))
    close(got, ref)
    with pytest.raises(ValueError):
        moe.decode(O.make_tokens(17).to(cuda), pg["w_gu"], pg["w_d"], torch.zeros(17, 8, dtype=torch.long, device=cuda),
                   torch.zeros(17, 8, device=cuda))


@pytest.mark.parametrize("M", [1, 2, 4, 8, 16])
@pytest.mark.parametrize("seed", [0, 3])
def test_block_decode_fused_router_bf16(cuda, base_params, M, seed):
    """One kernel: RMSNorm + softmax top-6 router + 6 routed + 2 shared slots + residual."""
    from mingmoe.block import MoeBlock
    p = base_params
    blk = MoeBlock.from_params(p)
    x = O.make_tokens(M, seed=seed)
    y_ref, ids_ref, wts_ref, _ = O.moe_block(x, p, top_k=6)
    logits = torch.empty(M, 64, device=cuda)
    ids = torch.empty(M, 8, dtype=torch.long, device=cuda)
    wts = torch.empty(M, 8, device=cuda)
    y = blk.decode(x.to(cuda), logits=logits, ids=ids, wts=wts)
    assert torch.equal(ids.cpu(), ids_ref)
    assert torch.allclose(wts.cpu(), wts_ref, rtol=2e-7, atol=0)
    close(y, y_ref)
    no_device_errors()
    # repeated calls (the kernel leaves its workspace zeroed: barrier counters reset)
    for _ in range(3):
        y2 = blk.decode(x.to(cuda))
    assert torch.equal(y2, y)


@pytest.mark.parametrize("M", [1, 4, 16])
def test_block_decode_int8(cuda, int8_params, M):
    from mingmoe.block import MoeBlock
    p = int8_params
    blk = MoeBlock.from_params(p)
    x = O.make_tokens(M, seed=1)
    y_ref, ids_ref, _, _ = O.moe_block(x, p, top_k=6)
    ids = torch.empty(M, 8, dtype=torch.int32, device=cuda)
    y = blk.decode(x.to(cuda), ids=ids)
    assert torch.equal(ids.cpu().long(), ids_ref)
    close(y, y_ref)
    no_device_errors()


@pytest.mark.parametrize("int8,M", [(False, 2), (True, 2), (True, 5)])
def test_block_decode_per_token_launches_match_single_tokens(cuda, base_params, int8_params, int8, M):
    """bf16 M = 2 and int8 M >= 2 run the one-token kernel once per token: the rows, ids, weights and logits of
    one M-token call are bitwise those of M one-token calls."""
    from mingmoe.block import MoeBlock
    blk = MoeBlock.from_params(int8_params if int8 else base_params)
    x = O.make_tokens(M, seed=11).to(cuda)
    ids = torch.empty(M, 8, dtype=torch.long, device=cuda)
    wts = torch.empty(M, 8, device=cuda)
    logits = torch.empty(M, 64, device=cuda)
    y = blk.decode(x, logits=logits, ids=ids, wts=wts).clone()
    for t in range(M):
        ids1 = torch.empty(1, 8, dtype=torch.long, device=cuda)
        wts1 = torch.empty(1, 8, device=cuda)
        logits1 = torch.empty(1, 64, device=cuda)
        y1 = blk.decode(x[t:t + 1].contiguous(), logits=logits1, ids=ids1, wts=wts1)
        assert torch.equal(y1, y[t:t + 1])
        assert torch.equal(ids1, ids[t:t + 1]) and torch.equal(wts1, wts[t:t + 1])
        assert torch.equal(logits1, logits[t:t + 1])
    no_device_errors()


def test_block_decode_sigmoid_group_reference_model(cuda):
    """ming-voice's own router (sigmoid + bias, 8 groups keep 4, top-8, x2.5) with its shared expert in slot E."""
    from mingmoe.block import MoeBlock
    g = torch.Generator().manual_seed(11)
    E, H, I = 128, 1536, 512
    p = O.make_block_params(seed=11, H=H, I=I, E=E, I_s=I)
    p.update(router_w=p["router_w"].float(), router_bias=torch.randn(E, generator=g) * 0.05, n_group=8,
             topk_group=4, scale=2.5)
    blk = MoeBlock.from_params(p, route_mode="sigmoid_group", top_k=8, router_bias=p["router_bias"])
    for M in (1, 3):
        x = O.make_tokens(M, H=H, seed=11)
        y_ref, ids_ref, wts_ref, _ = O.moe_block(x, p, top_k=8, router="sigmoid_group")
        ids = torch.empty(M, 9, dtype=torch.long, device=cuda)
        wts = torch.empty(M, 9, device=cuda)
        y = blk.decode(x.to(cuda), ids=ids, wts=wts)
        assert torch.equal(ids.cpu(), ids_ref)
        assert torch.allclose(wts.cpu(), wts_ref, rtol=2e-7, atol=0)
        close(y, y_ref)
    no_device_errors()


@pytest.mark.parametrize("N", [17, 40])
def test_block_prefill_small(cuda, base_params, N):
    from mingmoe.block import MoeBlock
    p = base_params
    blk = MoeBlock.from_params(p)
    x = O.make_tokens(N, seed=5)
    y_ref, _, _, _ = O.moe_block(x, p, top_k=6)
    close(blk.prefill(x.to(cuda)), y_ref)
    no_device_errors()


@pytest.mark.parametrize("M", [1, 5, 16])
def test_decode_tensor_core_and_cuda_core_paths_agree(cuda, base_params, M):
    """MINGMOE_DECODE_PATH=tc / =classic force the tcgen05 or the CUDA-core kernel: both match the oracle."""
    import os
    from mingmoe.block import MoeBlock
    p = base_params
    blk = MoeBlock.from_params(p)
    x = O.make_tokens(M, seed=40 + M).to(cuda)
    y_ref, ids_ref, _, _ = O.moe_block(x.cpu(), p, top_k=6)
    os.environ["MINGMOE_DECODE_PATH"] = "tc"
    try:
        ids_tc = torch.empty(M, 8, dtype=torch.long, device=cuda)
        y_tc = blk.decode(x, ids=ids_tc)
    finally:
        del os.environ["MINGMOE_DECODE_PATH"]
    os.environ["MINGMOE_DECODE_PATH"] = "classic"
    try:
        ids_cc = torch.empty(M, 8, dtype=torch.long, device=cuda)
        y_cc = blk.decode(x, ids=ids_cc)
    finally:
        del os.environ["MINGMOE_DECODE_PATH"]
    assert torch.equal(ids_tc, ids_cc) and torch.equal(ids_tc.cpu(), ids_ref)
    close(y_tc, y_ref)
    close(y_cc, y_ref)
    close(y_tc, y_cc.float(), max_abs=1.6e-2)
    no_device_errors()


@pytest.mark.parametrize("M", [1, 3, 16])
def test_decode_skips_pairs_marked_minus_one(cuda, base_params, base_params_gpu, M):
    """Expert-parallel prefill marks the pairs held by another rank with id -1; with <= 16 tokens they reach the
    decode kernels, which skip them without flagging an error (an id outside [0, E1) other than -1 is flagged)."""
    p, pg = base_params, base_params_gpu
    x = O.make_tokens(M, seed=9)
    xn = O.rms_norm(x, p["norm_w"], p["eps"])
    ids, wts, _ = O.route_softmax(xn, p["router_w"], top_k=6, shared_ids=p["shared_ids"])
    ids = ids.clone()
    ids[:, 1::2] = -1  # every other pair lives elsewhere
    ref = O.moe_experts(xn, p["w_gu"], p["w_d"], torch.where(ids < 0, 0, ids), torch.where(ids < 0, 0.0, wts))
    L.all_workspace_errors(clear=True)
    for path in ("c", "tc"):
        import os
        os.environ["MINGMOE_DECODE_PATH"] = path
        try:
            got = moe.experts(xn.to(cuda), pg["w_gu"], pg["w_d"], ids.to(cuda).to(torch.int32), wts.to(cuda))
        finally:
            del os.environ["MINGMOE_DECODE_PATH"]
        close(got, ref)
        no_device_errors()
