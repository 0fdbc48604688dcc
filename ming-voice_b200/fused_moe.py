"""Drop-in replacement for ming-voice's fused_moe.py, backed by the sm_100a kernels of libmingmoe
(include/mingmoe.h). Same names, arguments and return conventions:

  fused_moe_decode(x, w_gu, w_d, ids, weights, a_buf=None, out=None, s_gu=None, s_d=None)   fused_moe.py:67
  fused_moe_prefill(x, w_gu, w_d, ids, weights, s_gu=None, s_d=None)                        fused_moe.py:176
  quantize_rows_int8(w)                                                                     fused_moe.py:199
  CFG, GCFG                                                                                 fused_moe.py:64, :151

Experts (plus the shared expert slot(s)) live in stacked tensors w_gu [E1, 2I, H] (gate rows then up rows)
and w_d [E1, H, I], bf16, or int8 with per-output-row scales s_gu [E1, 2I] / s_d [E1, H] (fp32 as the
reference stores them, or bf16).

Differences from the reference, all within its tolerance contract: gate/up/activation/per-expert outputs stay
fp32 instead of being rounded to bf16 (the output is rounded once); ragged tiles are handled (the reference
reads out of bounds when BK does not divide I, e.g. I=1408 with BK=256).
"""
from __future__ import annotations

import torch

from mingmoe import _lib as L
from mingmoe import moe as _moe

# Tile configs of the reference Triton kernels. Kept because callers and tests assign them
# (dev/test_moe_prefill.py:57-68); the CUDA kernels choose their own tiling and ignore them.
CFG = dict(A=dict(BN=16, BK=256, num_warps=4), B=dict(BN=16, BK=256, num_warps=4))
GCFG = dict(A=dict(BM=32, BN=32, BK=128, num_warps=4), B=dict(BM=32, BN=64, BK=64, num_warps=4))


def fused_moe_decode(x, w_gu, w_d, ids, weights, a_buf=None, out=None, s_gu=None, s_d=None):
    """x: [1, H] bf16 (or [M, H] with M <= 16); ids: [NK] int (or [M, NK]); weights: [NK] fp32 (shared expert
    weight 1.0 included). Returns y [1, H] bf16 = sum_k weights[k] * expert_{ids[k]}(x) (written into `out`
    when given). `a_buf` is accepted for compatibility and not used: the kernel keeps the activations on chip."""
    H = x.shape[-1]
    x2 = x.reshape(-1, H)
    M = x2.shape[0]
    y = torch.empty(M, H, device=x.device, dtype=torch.bfloat16) if out is None else out
    _moe.decode(x2, w_gu, w_d, ids.reshape(M, -1), weights.reshape(M, -1), out=y.view(M, H), s_gu=s_gu, s_d=s_d)
    return y


def fused_moe_prefill(x, w_gu, w_d, ids, weights, s_gu=None, s_d=None):
    """x: [N, H] bf16; ids: [N, K+1] expert ids per token (shared expert included); weights: [N, K+1] fp32.
    Returns [N, H] x.dtype = sum_k weights[:, k] * expert_k(x)."""
    N, H = x.shape
    ids2 = ids.reshape(N, -1)
    w2 = weights.reshape(N, -1)
    return _moe.experts(x, w_gu, w_d, ids2, w2, s_gu=s_gu, s_d=s_d).to(x.dtype)


def quantize_rows_int8(w, scale_dtype=torch.float32):
    """Symmetric per-output-row int8: w [..., N, K] -> (int8 [..., N, K], scales [..., N]) with
    scale = max|w| / 127 (fp32 by default, as the reference; bf16 with scale_dtype=torch.bfloat16) and
    q = round_half_even(w / scale) clamped to +-127. Bit-exact with the reference's torch code."""
    L.require_cuda(w)
    K = w.shape[-1]
    w2 = w.reshape(-1, K)
    if w2.stride(-1) != 1:
        w2 = w2.contiguous()
    q = torch.empty(w.shape, dtype=torch.int8, device=w.device)
    s = torch.empty(w.shape[:-1], dtype=scale_dtype, device=w.device)
    L.check(L.lib().mv_quantize_rows_int8(L.ptr(w2), L.dt(w2), w2.stride(0), w2.shape[0], K, L.ptr(q), L.ptr(s),
                                          L.dt(s), L.stream_ptr(w.device)), "quantize_rows_int8")
    return q, s


def dequantize_rows_int8(q, scale):
    """float(q) * float(scale) per row, computed by the same device function the int8 kernels use."""
    L.require_cuda(q, scale)
    K = q.shape[-1]
    q2 = q.reshape(-1, K).contiguous()
    out = torch.empty(q.shape, dtype=torch.float32, device=q.device)
    L.check(L.lib().mv_dequant_rows_int8(L.ptr(q2), L.ptr(scale.contiguous()), L.dt(scale), q2.shape[0], K,
                                         L.ptr(out), L.stream_ptr(q.device)), "dequantize_rows_int8")
    return out
