"""Drop-in for ming-voice's `fastlinear.py` (small-M linear layers of the Talker step and the shared expert).

small_linear(x, w, b=None, act=0, residual=None, out=None, norm=None) keeps the reference's signature and
semantics (fastlinear.py:142-174): up to 16 rows run through mv_small_linear (one sm_100a kernel, fused RMSNorm
prologue, bias / gelu-tanh / silu / residual epilogue); more rows take the same torch path the reference takes.
The reference autotunes a Triton config per shape and caches it on disk; the CUDA kernel needs no tuning, so
save_cache() has nothing to save and small_linear never raises for an untuned shape during graph capture.
"""
from __future__ import annotations

import ctypes as C

import torch

from mingmoe import _lib as L


def save_cache():
    """Kept for the reference's callers (server warm-up): there is no per-shape tuning state to persist."""
    return None


def _graph_time(fn, reps=20, inner=40):
    """Seconds per call of fn (same name and arguments as the reference's helper, fastlinear.py:105-122, which
    dev/mm_compare.py imports). One CUDA graph holds `inner` calls; after one warm replay, `reps` replays are
    bracketed by CUDA events on the replay stream, so the figure is device time without host launch cost."""
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(side):
        fn()  # creates any lazily built state (workspaces) outside the capture
        with torch.cuda.graph(graph, stream=side):
            for _ in range(inner):
                fn()
        graph.replay()
        begin, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        begin.record(side)
        for _ in range(reps):
            graph.replay()
        end.record(side)
    end.synchronize()
    torch.cuda.current_stream().wait_stream(side)
    return begin.elapsed_time(end) * 1e-3 / (reps * inner)


def small_linear(x, w, b=None, act=0, residual=None, out=None, norm=None):
    """x: [..., K] with prod(leading) <= 16; w: [N, K] contiguous; act: 0 none, 1 gelu-tanh, 2 silu;
    residual: [..., N] added after the activation; norm: (gamma, eps) applies RMSNorm to x first (fused)."""
    shape = x.shape
    x2 = x.reshape(-1, shape[-1])
    if not x2.is_contiguous():
        x2 = x2.contiguous()
    M, N, K = x2.shape[0], w.shape[0], x2.shape[1]
    if M > 16:
        if norm is not None:
            x2 = torch.nn.functional.rms_norm(x2, (K,), norm[0], norm[1])
        y = torch.nn.functional.linear(x2, w, b)
        if act == 1:
            y = torch.nn.functional.gelu(y, approximate="tanh")
        elif act == 2:
            y = torch.nn.functional.silu(y)
        y = y.reshape(*shape[:-1], N)
        return y + residual if residual is not None else y
    L.require_cuda(x2, w, b, residual)
    if x2.dtype != torch.bfloat16 or w.dtype != torch.bfloat16:
        raise TypeError("small_linear: x and w must be bf16")
    if w.stride(1) != 1:
        raise ValueError("small_linear: w must have a unit inner stride")
    r2 = None
    if residual is not None:
        r2 = residual.reshape(-1, N)
        if not r2.is_contiguous():
            r2 = r2.contiguous()
    g, eps = (norm[0].contiguous(), float(norm[1])) if norm is not None else (None, 0.0)
    bb = b.contiguous() if b is not None else None
    y = torch.empty(M, N, device=x.device, dtype=x.dtype) if out is None else out.reshape(M, N)
    L.check(L.lib().mv_small_linear(L.ptr(x2), x2.stride(0), L.ptr(w), w.stride(0), L.ptr(bb), L.ptr(r2),
                                    r2.stride(0) if r2 is not None else 0, L.ptr(g), C.c_float(eps), int(act),
                                    L.ptr(y), y.stride(0), M, N, K, L.stream_ptr(x.device)), "mv_small_linear")
    return y.reshape(*shape[:-1], N)
