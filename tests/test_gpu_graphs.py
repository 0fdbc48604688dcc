"""CUDA-graph replay of the block against the fp32 oracle: the decode step of a layer stack (bf16 at M = 1 and 16,
int8 at M = 1), a captured prefill pass (also after a larger eager prefill on the capture stream has outgrown the
workspace the graph uses), and the padded-bucket prefill graphs. ming-voice's decode step and short-prompt
prefill are graph replays (engine.py:694-757, replay at :950-961 and :980), so this is the path that runs.

Tolerance: router ids bit-exact; bf16 outputs within max-abs 2e-2 and mean-rel 1e-2 of
the fp32 oracle, mean-rel being sum|got - ref| / sum|ref|."""
import pytest
import torch

from mingmoe import _lib as L
from mingmoe.block import MoeBlock
from mingmoe.graphs import DecodeGraph, PrefillGraphs
from oracle import moe_oracle as O

pytestmark = pytest.mark.gpu

MAX_ABS, MEAN_REL = 2e-2, 1e-2
LAYERS = 3


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


def check_stack(g, x, p):
    """Each block of a replayed stack against the oracle block applied to that block's own input (the token for
    block 0, the GPU stack's bf16 output of block l - 1 for block l): the BASELINE tolerance is per block, and
    compounding it over layers would test the tolerance, not the kernels."""
    h = x
    for layer in range(len(g.bufs)):
        y_ref, ids_ref, _, _ = O.moe_block(h, p, top_k=6)
        assert torch.equal(g.ids[layer].cpu().long(), ids_ref), layer
        close(g.bufs[layer], y_ref)
        h = g.bufs[layer].cpu()


@pytest.fixture(scope="module")
def base_params():
    return O.make_block_params(seed=0)


@pytest.fixture(scope="module")
def int8_params():
    return O.make_block_params(seed=1, int8=True)


def stack_of(p, layers, link=True, router_bias=None):
    blocks = [MoeBlock.from_params(p, router_bias=router_bias) for _ in range(layers)]
    if link:
        for i, b in enumerate(blocks):
            b.link(blocks[(i + 1) % layers])
    return blocks


@pytest.mark.parametrize("M", [1, 16])
def test_decode_graph_stack_bf16(cuda, base_params, M):
    blocks = stack_of(base_params, LAYERS)
    g = DecodeGraph(blocks, M)
    x = O.make_tokens(M, seed=40 + M)
    first = None
    for _ in range(3):
        g.ids.zero_()
        y = g(x.to(cuda))
        torch.cuda.synchronize()
        if first is None:
            check_stack(g, x, base_params)
            first = y.clone()
        assert torch.equal(y, first)  # replays are deterministic
    no_device_errors()


def test_decode_graph_stack_int8(cuda, int8_params):
    blocks = stack_of(int8_params, LAYERS)
    g = DecodeGraph(blocks, 1)
    x = O.make_tokens(1, seed=77)
    first = None
    for _ in range(3):
        y = g(x.to(cuda))
        torch.cuda.synchronize()
        if first is None:
            check_stack(g, x, int8_params)
            first = y.clone()
        assert torch.equal(y, first)
    no_device_errors()


def test_prefill_graph_survives_workspace_growth(cuda, base_params):
    """A captured prefill pass keeps its workspace: a larger eager prefill on the capture stream moves later calls
    to a bigger buffer but must not free the one the graph writes to."""
    bias = O.zipf_bias(64)
    blk = MoeBlock.from_params(base_params, router_bias=bias)
    N = 300
    x = O.make_tokens(N, seed=5)
    ref, _, _, _ = O.moe_block(x, base_params, top_k=6, bias=bias)
    xs = x.to(cuda)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(2):
            blk.prefill(xs)
        s.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            y = blk.prefill(xs)
        for _ in range(3):
            g.replay()
            s.synchronize()
            close(y, ref)
        big = O.make_tokens(2043, seed=6).to(cuda)
        before = len(L._retired)
        blk.prefill(big)  # grows the prefill / route / align workspaces of stream s
        s.synchronize()
        assert len(L._retired) > before
        torch.cuda.empty_cache()
        junk = torch.full((64 << 20,), 0x7f, dtype=torch.uint8, device=cuda)  # reuse freed memory if any
        g.replay()
        s.synchronize()
        close(y, ref)
        del junk
    torch.cuda.current_stream().wait_stream(s)
    no_device_errors()


def test_prefill_bucket_graphs(cuda, base_params):
    """Each prompt length replays the graph of the smallest bucket holding it (longer ones run eagerly)."""
    pg = PrefillGraphs([MoeBlock.from_params(base_params)], buckets=(32, 64, 128))
    for T in (1, 7, 32, 33, 100, 128, 150):
        x = O.make_tokens(T, seed=100 + T)
        ref, _, _, _ = O.moe_block(x, base_params, top_k=6)
        y = pg(x.to(cuda))
        torch.cuda.synchronize()
        assert y.shape == (T, 2048)
        close(y, ref)
    no_device_errors()


def test_prefill_bucket_graphs_stack(cuda, base_params):
    """A two-block stack in one bucket graph gives what the two blocks give eagerly on the same padded rows."""
    blocks = stack_of(base_params, 2, link=False)
    pg = PrefillGraphs(blocks, buckets=(64,))
    x = O.make_tokens(50, seed=3).to(cuda)
    y = pg(x).clone()
    h = x
    for blk in blocks:
        h = blk.prefill(h)
    torch.cuda.synchronize()
    d = (y.float() - h.float()).abs()
    # both run the same kernels; only the fp32 reduction order of the down projection differs, so the outputs
    # agree to about one bf16 step of the result's magnitude
    assert (d.sum() / h.float().abs().sum()).item() <= 1e-3
    assert d.max().item() <= 2 * torch.finfo(torch.bfloat16).eps * h.float().abs().max().item()
    no_device_errors()


def test_mask_pad_rows(cuda):
    for dt in (torch.int32, torch.int64):
        ids = torch.arange(40 * 8, device=cuda).reshape(40, 8).to(dt)
        n = torch.tensor([13], dtype=torch.int32, device=cuda)
        L.check(L.lib().mv_mask_pad_rows(L.ptr(ids), L.dt(ids), 40, 8, L.ptr(n), L.stream_ptr(cuda)), "mask")
        torch.cuda.synchronize()
        want = torch.arange(40 * 8).reshape(40, 8)
        want[13:] = -1
        assert torch.equal(ids.cpu().long(), want)
