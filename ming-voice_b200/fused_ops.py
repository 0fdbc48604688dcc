"""Drop-in replacement for ming-voice's fused_ops.py (RMSNorm + MoE router), backed by the sm_100a kernels of
libmingmoe (include/mingmoe.h). Same function names, argument meaning and in-place output convention.

  rms_norm(x, w, eps)                        fused_ops.py:28-37
  moe_route(x, w32, bias, n_group, topk_group, top_k, scale, logits_buf, ids_out, wts_out)
                                             fused_ops.py:96-103 (sigmoid + group-limited top-k); extended to
                                             n tokens, and with mode="softmax" to the BASELINE router
"""
from __future__ import annotations

import torch

from mingmoe import _lib as L


def rms_norm(x, w, eps):
    """BailingMoeV3RMSNorm: fp32 statistics, normalise, cast to x.dtype, scale by w; output dtype
    promote(w.dtype, x.dtype) (fused_ops.py:33-34)."""
    L.require_cuda(x, w)
    N = x.shape[-1]
    x2 = x.reshape(-1, N)
    if not x2.is_contiguous():
        x2 = x2.contiguous()
    out_dtype = torch.promote_types(w.dtype, x.dtype)
    y = torch.empty(x2.shape, dtype=out_dtype, device=x.device)
    L.check(L.lib().mv_rmsnorm(L.ptr(x2), L.dt(x2), x2.stride(0), L.ptr(w.contiguous()), L.dt(w), L.ptr(y), L.dt(y),
                               x2.shape[0], N, float(eps), L.stream_ptr(x.device)), "rms_norm")
    return y.view(x.shape)


def moe_route(x, w32, bias, n_group, topk_group, top_k, scale, logits_buf, ids_out, wts_out, *, mode="sigmoid_group",
              n_shared=1, shared_id=None, w_scale=None):
    """Router for the tokens of x ([1, H] as in the reference, or [n, H]). Writes in place:
    logits_buf [n*E] fp32, ids_out [n*(top_k+n_shared)] (dtype taken from ids_out, int64 in the engine),
    wts_out [same] fp32: the top_k experts (largest first, ties to the lower id) followed by the shared
    slot(s) shared_id.. (default E) with weight 1.0. Returns (ids_out, wts_out, logits_buf).

    mode="sigmoid_group" (the reference, fused_ops.py:53-93): sigmoid scores + bias, keep `topk_group` of
    `n_group` groups by their top-2 sum, top_k, weights renormalised (+1e-20) times `scale`.
    mode="softmax" (BASELINE): softmax over logits (+ bias), top_k, renormalised; n_group/topk_group/scale
    ignored. w32 may be fp32, bf16, or int8 with `w_scale`."""
    L.require_cuda(x, w32)
    E, H = w32.shape
    x2 = x.reshape(-1, H)
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    if x2.dtype != torch.bfloat16:
        raise TypeError("moe_route: x must be bf16")
    n = x2.shape[0]
    sid = E if shared_id is None else int(shared_id)
    nkt = top_k + n_shared
    if ids_out.numel() != n * nkt or wts_out.numel() != n * nkt:
        raise ValueError(f"moe_route: ids_out/wts_out need {n * nkt} elements")
    if logits_buf is not None and logits_buf.numel() != n * E:
        raise ValueError(f"moe_route: logits_buf needs {n * E} elements")
    if wts_out.dtype != torch.float32 or (logits_buf is not None and logits_buf.dtype != torch.float32):
        raise TypeError("moe_route: wts_out and logits_buf must be fp32")
    for t in (ids_out, wts_out, logits_buf):
        if t is not None and not t.is_contiguous():
            raise ValueError("moe_route: output buffers must be contiguous")
    m = L.MV_ROUTE_SIGMOID_GROUP if mode == "sigmoid_group" else L.MV_ROUTE_SOFTMAX
    if mode not in ("sigmoid_group", "softmax"):
        raise ValueError(f"moe_route: unknown mode {mode!r}")
    w = w32 if w32.is_contiguous() else w32.contiguous()
    b = None
    if bias is not None:
        b = bias.float().contiguous()
    ws = L.workspace("route", L.lib().mv_route_workspace_bytes(n, E), x.device)
    L.check(L.lib().mv_route(m, L.ptr(x2), x2.stride(0), L.ptr(w), L.dt(w), L.ptr(w_scale),
                             L.dt(w_scale) if w_scale is not None else L.MV_F32, L.ptr(b), n, H, E, int(top_k),
                             int(n_group), int(topk_group), float(scale), int(n_shared), sid, L.ptr(logits_buf),
                             L.ptr(ids_out), L.dt(ids_out), L.ptr(wts_out), L.ptr(ws), ws.numel(),
                             L.stream_ptr(x.device)), "moe_route")
    return ids_out, wts_out, logits_buf


def route_softmax(x, w, top_k, bias=None, n_shared=0, shared_id=None, w_scale=None, ids_dtype=torch.int64):
    """BASELINE router convenience: allocates the outputs. Returns (ids [n, top_k+n_shared], wts fp32,
    logits [n, E] fp32)."""
    E, H = w.shape
    n = x.reshape(-1, H).shape[0]
    ids = torch.empty(n, top_k + n_shared, dtype=ids_dtype, device=x.device)
    wts = torch.empty(n, top_k + n_shared, dtype=torch.float32, device=x.device)
    logits = torch.empty(n, E, dtype=torch.float32, device=x.device)
    moe_route(x, w, bias, 1, 1, top_k, 1.0, logits, ids, wts, mode="softmax", n_shared=n_shared,
              shared_id=E if shared_id is None else shared_id, w_scale=w_scale)
    return ids, wts, logits
