"""Multi-token (prefill) expert path for N > 16 tokens.

Until the grouped tensor-core path is in place, tokens go through the decode kernel 16 at a time (a GPU path
with the same numerics, not a fallback to PyTorch)."""
from __future__ import annotations

import torch

from . import moe


def experts(x, w_gu, w_d, ids, wts, s_gu=None, s_d=None, out=None, residual=None):
    N, H = x.shape
    y = torch.empty(N, H, dtype=torch.bfloat16, device=x.device) if out is None else out
    for n0 in range(0, N, moe.DECODE_MAX_M):
        n1 = min(N, n0 + moe.DECODE_MAX_M)
        moe.decode(x[n0:n1], w_gu, w_d, ids[n0:n1], wts[n0:n1], out=y[n0:n1], s_gu=s_gu, s_d=s_d,
                   residual=None if residual is None else residual[n0:n1])
    return y
