"""mv_block_decode_noalloc (static device scratch, no workspace argument) against mv_block_decode.

Collected last (file name) so that it also runs after every other test in one process; it passes alone too."""
import ctypes as C

import pytest
import torch

from mingmoe import _lib as L
from mingmoe.block import MoeBlock
from oracle import moe_oracle as O

pytestmark = pytest.mark.gpu

MAX_ABS, MEAN_REL = 2e-2, 1e-2


def call_noalloc(blk, x, out, ids, wts, status):
    return L.lib().mv_block_decode_noalloc(C.byref(blk._block), L.ptr(x), x.shape[0], L.ptr(out), None, L.ptr(ids),
                                           L.dt(ids), L.ptr(wts), L.ptr(status), L.stream_ptr(x.device))


@pytest.mark.parametrize("M", [1, 4, 16])
def test_noalloc_matches_workspace_entry_point(cuda, M):
    p = O.make_block_params(seed=0)
    blk = MoeBlock.from_params(p)
    x = O.make_tokens(M, seed=21).to(cuda)
    ids_ref = torch.empty(M, 8, dtype=torch.long, device=cuda)
    wts_ref = torch.empty(M, 8, device=cuda)
    y_ref = blk.decode(x, ids=ids_ref, wts=wts_ref)
    for _ in range(2):  # two calls in a row reuse the one static scratch
        out = torch.empty_like(x)
        ids = torch.full((M, 8), -1, dtype=torch.long, device=cuda)
        wts = torch.zeros(M, 8, device=cuda)
        status = torch.full((2,), 7, dtype=torch.int32, device=cuda)
        rc = call_noalloc(blk, x, out, ids, wts, status)
        assert rc == 0, L.lib().mv_last_error().decode()
        torch.cuda.synchronize()
        assert torch.equal(ids, ids_ref)
        assert torch.equal(wts, wts_ref)
        d = (out.float() - y_ref.float()).abs()
        assert d.max().item() <= MAX_ABS
        assert (d.sum() / y_ref.float().abs().sum()).item() <= MEAN_REL
        assert status.tolist() == [0, 0]


def test_noalloc_alternating_token_counts(cuda):
    """Calls with different M in a row on one stream: each finds the shared scratch as a call of another token
    count (another instance of the CUDA-core kernel: 1, up to 4 or up to 16 tokens) left it. Within the 1 MiB
    scratch every call runs the CUDA-core kernel; the reference calls below, with a full workspace, run the
    tensor-core kernel from M = 2, so the two agree within the tolerance, not bit for bit."""
    p = O.make_block_params(seed=0)
    blk = MoeBlock.from_params(p)
    for M in (16, 1, 4, 1, 2, 16, 8, 1):
        x = O.make_tokens(M, seed=30 + M).to(cuda)
        ids_ref = torch.empty(M, 8, dtype=torch.long, device=cuda)
        y_ref = blk.decode(x, ids=ids_ref)
        out = torch.empty_like(x)
        ids = torch.full((M, 8), -1, dtype=torch.long, device=cuda)
        wts = torch.zeros(M, 8, device=cuda)
        status = torch.full((2,), 7, dtype=torch.int32, device=cuda)
        assert call_noalloc(blk, x, out, ids, wts, status) == 0, L.lib().mv_last_error().decode()
        torch.cuda.synchronize()
        assert torch.equal(ids, ids_ref), M
        d = (out.float() - y_ref.float()).abs()
        assert d.max().item() <= MAX_ABS
        assert (d.sum() / y_ref.float().abs().sum()).item() <= MEAN_REL
        assert status.tolist() == [0, 0], M


def test_noalloc_rejects_scratch_beyond_its_size(cuda):
    b = L.Block()
    b.E, b.top_k, b.n_shared = 64, 6, 2
    b.experts.I, b.experts.H, b.experts.E1 = 2048, 2048, 66  # 16 x 8 x 2048 x 4 B of activations > 1 MiB
    x = torch.zeros(16, 2048, dtype=torch.bfloat16, device=cuda)
    rc = L.lib().mv_block_decode_noalloc(C.byref(b), L.ptr(x), 16, L.ptr(x), None, None, L.MV_I64, None, None,
                                         L.stream_ptr(x.device))
    assert rc == 5  # MV_ERR_WORKSPACE
    assert "static scratch holds 1048576" in L.lib().mv_last_error().decode()
