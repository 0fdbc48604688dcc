"""Multi-token (prefill) expert path: expert-sorted grouped GEMMs on the tensor cores (mv_moe_prefill).

bf16 and int8 weights both take the tcgen05 path (int8: the experts in use are widened to bf16 exactly and the
row scales multiply the fp32 products, the reference's int8 numerics, fused_moe.py:115-121)."""
from __future__ import annotations

import ctypes as C

import torch

from . import _lib as L
from . import moe


def align(ids: torch.Tensor, E1: int, BM: int):
    """fused_moe._align_blocks (fused_moe.py:154-173) on the GPU: (sorted_ids, bexp, nb_used)."""
    L.require_cuda(ids)
    flat = ids.reshape(-1)
    if not flat.is_contiguous():
        flat = flat.contiguous()
    P = flat.numel()
    nb_max = (P + E1 * (BM - 1) + BM - 1) // BM
    sorted_ids = torch.empty(nb_max * BM, dtype=torch.int32, device=ids.device)
    bexp = torch.empty(nb_max, dtype=torch.int32, device=ids.device)
    nb_used = torch.empty(1, dtype=torch.int32, device=ids.device)
    ws = L.workspace("align", L.lib().mv_moe_align_workspace_bytes(P, E1), ids.device)
    L.check(L.lib().mv_moe_align(L.ptr(flat), L.dt(flat), P, E1, BM, L.ptr(sorted_ids), L.ptr(bexp), L.ptr(nb_used),
                                 L.ptr(ws), ws.numel(), L.stream_ptr(ids.device)), "mv_moe_align")
    return sorted_ids, bexp, nb_used


def experts(x, w_gu, w_d, ids, wts, s_gu=None, s_d=None, out=None, residual=None):
    N, H = x.shape
    y = torch.empty(N, H, dtype=torch.bfloat16, device=x.device) if out is None else out
    L.require_cuda(x)
    if x.dtype != torch.bfloat16:
        raise TypeError("prefill: x must be bf16")
    if x.stride(1) != 1:
        x = x.contiguous()
    ids2, wts2 = moe._ids_wts(ids, wts, N)
    NK = ids2.shape[1]
    wst = moe.weights_struct(w_gu, w_d, s_gu, s_d)
    E1, I = w_gu.shape[0], w_gu.shape[1] // 2
    nbytes = L.lib().mv_moe_prefill_workspace_bytes(N, NK, H, I, E1, L.dt(w_gu))
    ws = L.workspace("prefill", nbytes, x.device)
    r = residual
    if r is not None and r.stride(1) != 1:
        r = r.contiguous()
    L.check(L.lib().mv_moe_prefill(C.byref(wst), L.ptr(x), x.stride(0), L.ptr(ids2), L.dt(ids2), L.ptr(wts2), N, NK,
                                   L.ptr(r), r.stride(0) if r is not None else 0, L.ptr(y), L.ptr(ws), ws.numel(),
                                   L.stream_ptr(x.device)), "mv_moe_prefill")
    return y
