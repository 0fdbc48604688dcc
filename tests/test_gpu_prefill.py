"""GPU parity of the prefill path: the expert sort (bit-exact against the reference's _align_blocks
restatement and its golden vectors) and the tcgen05 grouped GEMMs (BASELINE tolerance against the fp32
oracle), at BASELINE dims (H=2048, I=1408, 64 experts + 2 shared slots, top-6) and ming-voice's own
(H=1536, I=512, 128 experts + 1 shared slot, top-8)."""
import numpy as np
import pytest
import torch

from conftest import golden
from mingmoe import _lib as L
from mingmoe import prefill
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


def check_align(flat, E1, BM):
    si, be, nb = O.align_blocks(flat.numpy(), E1, BM)
    for dt in (torch.int32, torch.int64):
        s, b, n = prefill.align(flat.to(dt).cuda(), E1, BM)
        torch.cuda.synchronize()
        assert np.array_equal(s.cpu().numpy(), si)
        assert np.array_equal(b.cpu().numpy(), be)
        used = int((be >= 0).sum())
        assert int(n.item()) == used
    assert nb == s.numel() // BM


def test_align_golden():
    d = golden("align_blocks")
    si, be, nb = O.align_blocks(d["flat"].numpy(), d["E1"], d["BM"])
    assert np.array_equal(si, d["sorted_ids"].numpy()) and np.array_equal(be, d["bexp"].numpy())
    check_align(d["flat"], d["E1"], d["BM"])
    no_device_errors()


@pytest.mark.parametrize("BM", [16, 32, 128])
def test_align_zipf_prefill_ids(BM):
    # the C4 router output shape: 2043 tokens x (6 routed + 2 shared), Zipf-skewed experts
    g = torch.Generator().manual_seed(2)
    logits = torch.randn(2043, 64, generator=g) + O.zipf_bias(64)
    top = torch.topk(logits, 6, dim=1).indices
    ids = torch.cat([top, torch.full((2043, 1), 64), torch.full((2043, 1), 65)], dim=1)
    check_align(ids.reshape(-1), 66, BM)
    # ragged extremes: one expert only, every expert once, a single pair
    check_align(torch.full((1000,), 3), 8, BM)
    check_align(torch.arange(300) % 300, 300, BM)
    check_align(torch.tensor([5]), 6, BM)
    no_device_errors()


@pytest.fixture(scope="module")
def base_params():
    return O.make_block_params(seed=0)


@pytest.fixture(scope="module")
def base_params_gpu(base_params):
    return {k: (v.cuda() if torch.is_tensor(v) else v) for k, v in base_params.items()}


@pytest.mark.parametrize("N", [1, 5, 17, 130, 300])
def test_prefill_experts_bf16(base_params, base_params_gpu, N):
    p, pg = base_params, base_params_gpu
    x = O.make_tokens(N, seed=N)
    xn = O.rms_norm(x, p["norm_w"], p["eps"])
    ids, wts, _ = O.route_softmax(xn, p["router_w"], top_k=6, shared_ids=p["shared_ids"])
    ref = O.moe_experts(xn, p["w_gu"], p["w_d"], ids, wts)
    got = prefill.experts(xn.cuda(), pg["w_gu"], pg["w_d"], ids.cuda(), wts.cuda())
    close(got, ref)
    got_r = prefill.experts(xn.cuda(), pg["w_gu"], pg["w_d"], ids.int().cuda(), wts.cuda(), residual=x.cuda())
    close(got_r, ref + x.float())
    no_device_errors()


def test_prefill_ragged_c4(base_params, base_params_gpu):
    """BASELINE C4: 4 packed sequences (37/211/512/1283 tokens), Zipf router bias, seed 2, full block."""
    from mingmoe.block import MoeBlock
    p = base_params
    bias = O.zipf_bias(64)
    blk = MoeBlock.from_params(p, router_bias=bias)
    N = sum(O.PREFILL_LENS)
    x = O.make_tokens(N, seed=2)
    y_ref, ids_ref, wts_ref, _ = O.moe_block(x, p, top_k=6, bias=bias)
    y = blk.prefill(x.cuda())
    close(y, y_ref)
    ids, wts, _ = blk.route(O.rms_norm(x, p["norm_w"], p["eps"]).cuda())
    assert torch.equal(ids.cpu().long(), ids_ref)
    no_device_errors()


def test_prefill_reference_model_dims():
    g = torch.Generator().manual_seed(13)
    E, H, I, N = 128, 1536, 512, 257
    w_gu = (torch.randn(E + 1, 2 * I, H, generator=g) * 0.02).to(torch.bfloat16)
    w_d = (torch.randn(E + 1, H, I, generator=g) * 0.02).to(torch.bfloat16)
    x = torch.randn(N, H, generator=g).to(torch.bfloat16)
    ids = torch.cat([torch.stack([torch.randperm(E, generator=g)[:8] for _ in range(N)]),
                     torch.full((N, 1), E)], dim=1)
    wts = torch.cat([torch.rand(N, 8, generator=g), torch.ones(N, 1)], dim=1)
    ref = O.moe_experts(x, w_gu, w_d, ids, wts)
    got = prefill.experts(x.cuda(), w_gu.cuda(), w_d.cuda(), ids.cuda(), wts.cuda())
    close(got, ref)
    no_device_errors()


def test_prefill_bad_id_flagged(base_params, base_params_gpu):
    p, pg = base_params, base_params_gpu
    x = O.make_tokens(40, seed=4)
    ids = torch.randint(0, 64, (40, 8), generator=torch.Generator().manual_seed(4))
    wts = torch.rand(40, 8, generator=torch.Generator().manual_seed(5))
    bad = ids.clone()
    bad[3, 2] = 999
    ref = O.moe_experts(x, p["w_gu"], p["w_d"], torch.where(bad == 999, 0, bad),
                        torch.where(bad == 999, torch.zeros_like(wts), wts))
    got = prefill.experts(x.cuda(), pg["w_gu"], pg["w_d"], bad.cuda(), wts.cuda())
    close(got, ref)
    errs = L.all_workspace_errors(clear=True)
    assert any(c == 2 for c, _ in errs.values())


@pytest.fixture(scope="module")
def int8_params():
    return O.make_block_params(seed=1, int8=True)


@pytest.mark.parametrize("N", [17, 300])
def test_prefill_experts_int8(int8_params, N):
    """BASELINE C3 weights (int8, bf16 scales) through the tcgen05 prefill: widened exactly, scaled in fp32."""
    p = int8_params
    pg = {k: (v.cuda() if torch.is_tensor(v) else v) for k, v in p.items()}
    x = O.make_tokens(N, seed=N + 1)
    xn = O.rms_norm(x, p["norm_w"], p["eps"])
    ids, wts, _ = O.route_softmax(xn, p["router_w"], top_k=6, shared_ids=p["shared_ids"], w_scale=p["router_s"])
    ref = O.moe_experts(xn, p["w_gu"], p["w_d"], ids, wts, s_gu=p["s_gu"], s_d=p["s_d"])
    got = prefill.experts(xn.cuda(), pg["w_gu"], pg["w_d"], ids.cuda(), wts.cuda(), s_gu=pg["s_gu"], s_d=pg["s_d"])
    close(got, ref)
    no_device_errors()


def test_prefill_block_int8_reference_model_fp32_scales():
    """ming-voice's own layout: H=1536, I=512, 128 experts + shared slot, fp32 row scales, sigmoid-group router."""
    from mingmoe.block import MoeBlock
    g = torch.Generator().manual_seed(21)
    E, H, I = 128, 1536, 512
    p = O.make_block_params(seed=21, H=H, I=I, E=E, I_s=I, int8=True, scale_dtype=torch.float32)
    # ming-voice keeps an fp32 copy of the gate (engine.py:324) next to int8 experts
    p["router_w"] = O.dequant_rows_int8(p["router_w"], p.pop("router_s"))
    p.update(router_bias=torch.randn(E, generator=g) * 0.05, n_group=8, topk_group=4, scale=2.5)
    blk = MoeBlock.from_params(p, route_mode="sigmoid_group", top_k=8, router_bias=p["router_bias"])
    x = O.make_tokens(150, H=H, seed=21)
    y_ref, _, _, _ = O.moe_block(x, p, top_k=8, router="sigmoid_group")
    close(blk.prefill(x.cuda()), y_ref)
    no_device_errors()


def test_prefill_skipped_pairs(base_params, base_params_gpu):
    """id -1 = a pair computed elsewhere (expert-parallel prefill): left out silently, the rest unchanged."""
    p, pg = base_params, base_params_gpu
    x = O.make_tokens(200, seed=9)
    g = torch.Generator().manual_seed(9)
    ids = torch.randint(0, 66, (200, 8), generator=g)
    wts = torch.rand(200, 8, generator=g)
    skip = torch.rand(200, 8, generator=g) < 0.3
    ref = O.moe_experts(x, p["w_gu"], p["w_d"], torch.where(skip, 0, ids), torch.where(skip, 0.0, wts))
    got = prefill.experts(x.cuda(), pg["w_gu"], pg["w_d"], torch.where(skip, -1, ids).int().cuda(), wts.cuda(),
                          residual=x.cuda())
    close(got, ref + x.float())
    no_device_errors()


def test_ep_prefill_one_rank():
    """The expert-parallel block on a world of one (NCCL): every pair local, output = the single-GPU block."""
    import os
    import socket
    import torch.distributed as dist
    from mingmoe.block import MoeBlock
    from mingmoe.ep import EPMoeBlock, shard_block_params
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("nccl", rank=0, world_size=1, device_id=torch.device("cuda", 0))
    try:
        p = O.make_block_params(seed=7, H=1024, I=512, E=16, I_s=1024)
        bias = O.zipf_bias(16)
        loc = shard_block_params(p, 0, 1, 16, replicated=(0, 1))
        ep = EPMoeBlock(MoeBlock.from_params(loc, router_bias=bias), 16, replicated=(0, 1))
        x = O.make_tokens(300, H=1024, seed=3)
        ref, _, _, _ = O.moe_block(x, p, top_k=6, bias=bias)
        close(ep.forward(x.cuda()), ref)
        no_device_errors()
    finally:
        dist.destroy_process_group()
