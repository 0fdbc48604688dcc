"""Host logic for the MoE expert kernels: argument marshalling into the C-ABI and regime dispatch.

decode()   M <= 16 tokens: one weight-streaming kernel (mv_moe_decode).
experts()  any N: N <= 16 goes to decode(); larger N goes to the grouped prefill path.
"""
from __future__ import annotations

import ctypes as C

import torch

from . import _lib as L

DECODE_MAX_M = 16


def weights_struct(w_gu, w_d, s_gu=None, s_d=None) -> L.MoeWeights:
    """Describe stacked expert tensors w_gu [E1, 2I, H], w_d [E1, H, I] (+ int8 row scales) for the C-ABI."""
    if w_gu.dim() != 3 or w_d.dim() != 3:
        raise ValueError("w_gu must be [E1, 2I, H] and w_d [E1, H, I]")
    E1, I2, H = w_gu.shape
    if w_d.shape[0] != E1 or w_d.shape[1] != H or 2 * w_d.shape[2] != I2:
        raise ValueError(f"inconsistent expert shapes {tuple(w_gu.shape)} / {tuple(w_d.shape)}")
    if w_gu.stride(2) != 1 or w_d.stride(2) != 1:
        raise ValueError("expert weights need a unit inner stride")
    if w_gu.dtype != w_d.dtype or w_gu.dtype not in (torch.bfloat16, torch.int8):
        raise TypeError("expert weights must both be bf16 or both int8")
    L.require_cuda(w_gu, w_d, s_gu, s_d)
    s = L.MoeWeights()
    s.w_gu, s.w_d = w_gu.data_ptr(), w_d.data_ptr()
    s.w_dtype = L.dt(w_gu)
    s.E1, s.H, s.I = E1, H, I2 // 2
    s.gu_se, s.gu_sr = w_gu.stride(0), w_gu.stride(1)
    s.d_se, s.d_sr = w_d.stride(0), w_d.stride(1)
    if w_gu.dtype == torch.int8:
        if s_gu is None or s_d is None:
            raise ValueError("int8 experts need s_gu and s_d")
        if s_gu.dtype != s_d.dtype or s_gu.dtype not in (torch.float32, torch.bfloat16):
            raise TypeError("scales must both be fp32 or both bf16")
        if s_gu.stride(-1) != 1 or s_d.stride(-1) != 1:
            raise ValueError("scales need a unit inner stride")
        s.s_gu, s.s_d = s_gu.data_ptr(), s_d.data_ptr()
        s.s_dtype = L.dt(s_gu)
        s.sgu_se, s.sd_se = s_gu.stride(0), s_d.stride(0)
    else:
        s.s_dtype = L.MV_F32
    return s


def _ids_wts(ids, wts, M):
    ids2 = ids.reshape(M, -1)
    if ids2.dtype not in (torch.int32, torch.int64):
        ids2 = ids2.long()
    ids2 = ids2.contiguous()
    w2 = wts.reshape(M, -1).float().contiguous()
    if w2.shape != ids2.shape:
        raise ValueError("ids and weights must have the same shape")
    return ids2, w2


def decode(x, w_gu, w_d, ids, wts, out=None, s_gu=None, s_d=None, norm_w=None, eps=1e-6, residual=None):
    """out[m] = bf16(residual[m] + sum_k wts[m,k] * expert_{ids[m,k]}(xn_m)), xn = RMSNorm(x) if norm_w."""
    L.require_cuda(x, ids, wts, residual, norm_w)
    M, H = x.shape
    if M > DECODE_MAX_M:
        raise ValueError(f"decode handles at most {DECODE_MAX_M} tokens, got {M}")
    if x.dtype != torch.bfloat16:
        raise TypeError("decode: x must be bf16")
    if x.stride(1) != 1:
        x = x.contiguous()
    ids2, w2 = _ids_wts(ids, wts, M)
    ws_w = weights_struct(w_gu, w_d, s_gu, s_d)
    y = torch.empty(M, H, dtype=torch.bfloat16, device=x.device) if out is None else out
    if residual is not None:
        residual = residual.reshape(M, H).contiguous()
    nbytes = L.lib().mv_moe_decode_workspace_bytes_tc(DECODE_MAX_M, max(ids2.shape[1], 16), ws_w.H, ws_w.I, ws_w.E1)
    ws = L.workspace("decode", nbytes, x.device)
    L.check(L.lib().mv_moe_decode(C.byref(ws_w), L.ptr(x), x.stride(0), L.ptr(norm_w), float(eps), L.ptr(ids2),
                                  L.dt(ids2), L.ptr(w2), M, ids2.shape[1], L.ptr(residual), L.ptr(y), L.ptr(ws),
                                  ws.numel(), L.stream_ptr(x.device)), "mv_moe_decode")
    return y


def experts(x, w_gu, w_d, ids, wts, s_gu=None, s_d=None, out=None, residual=None):
    """[residual +] sum_k wts[n,k] * expert_{ids[n,k]}(x_n) for N tokens, bf16 [N, H]."""
    N, H = x.shape
    if N <= DECODE_MAX_M:
        return decode(x, w_gu, w_d, ids, wts, out=out, s_gu=s_gu, s_d=s_d, residual=residual)
    from . import prefill
    return prefill.experts(x, w_gu, w_d, ids, wts, s_gu=s_gu, s_d=s_d, out=out, residual=residual)
