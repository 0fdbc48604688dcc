"""Quantise-on-load into the stacked expert layout.

ming-voice can keep its experts only as int8: the MoE blocks allocate `[E+1, 2I, H]` / `[E+1, H, I]` int8 stacks
and per-row scales, and the checkpoint loader routes every expert matrix to a hook that quantises it on the GPU
and copies it into its slot (engine.py:126-147), from several loader threads, each on its own CUDA stream
(direct_load.py:109-135). The hooks here have the same keys and call form (`hook(tensor)`), but each one is ONE
kernel (mv_quantize_into_stack) that writes the int8 rows and scales straight into the slot: no temporary
q / scale tensors, no copies. A source on the GPU or in pinned host memory is read in place; a pageable host
tensor is first copied into a per-thread staging buffer on the thread's current stream.
"""
from __future__ import annotations

import threading
from concurrent.futures import ThreadPoolExecutor

import torch

from . import _lib as L

_tls = threading.local()


def int8_stacks(E1: int, I: int, H: int, device, scale_dtype=torch.float32):
    """Empty int8 stacks in the reference layout: (q_gu [E1, 2I, H], s_gu [E1, 2I], q_d [E1, H, I], s_d [E1, H])."""
    q_gu = torch.empty(E1, 2 * I, H, dtype=torch.int8, device=device)
    q_d = torch.empty(E1, H, I, dtype=torch.int8, device=device)
    s_gu = torch.empty(E1, 2 * I, dtype=scale_dtype, device=device)
    s_d = torch.empty(E1, H, dtype=scale_dtype, device=device)
    return q_gu, s_gu, q_d, s_d


def _device_source(src: torch.Tensor, device) -> torch.Tensor:
    if src.is_cuda or src.is_pinned():
        return src if src.stride(-1) == 1 else src.contiguous()
    nbytes = src.numel() * src.element_size()
    key = torch.device(device).index or 0
    bufs = getattr(_tls, "staging", None)
    if bufs is None:
        bufs = _tls.staging = {}
    buf = bufs.get(key)
    if buf is None or buf.numel() < nbytes:
        buf = bufs[key] = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
    dst = buf[:nbytes].view(src.dtype).view(src.shape)
    dst.copy_(src)  # ordered on this thread's stream before the quantiser reads it
    return dst


def quantize_into(q_stack: torch.Tensor, s_stack: torch.Tensor, e: int, row_off: int, src: torch.Tensor):
    """Rows [row_off, row_off + n) of slot e of (q_stack [E1, R, K] int8, s_stack [E1, R]) from src [n, K]
    (bf16 / f16 / f32), on the current stream."""
    if q_stack.dtype != torch.int8 or not q_stack.is_contiguous() or not s_stack.is_contiguous():
        raise ValueError("quantize_into: contiguous int8 stack and scale stack required")
    E1, R, K = q_stack.shape
    if s_stack.shape != (E1, R):
        raise ValueError(f"quantize_into: scales {tuple(s_stack.shape)} do not match the stack {tuple(q_stack.shape)}")
    if src.dim() != 2 or src.shape[1] != K:
        raise ValueError(f"quantize_into: source {tuple(src.shape)} is not [n, {K}]")
    L.require_cuda(q_stack, s_stack)
    w = _device_source(src, q_stack.device)
    L.check(L.lib().mv_quantize_into_stack(L.ptr(w), L.dt(w), w.stride(0), w.shape[0], K, L.ptr(q_stack),
                                           L.ptr(s_stack), L.dt(s_stack), E1, R, int(e), int(row_off),
                                           L.stream_ptr(q_stack.device)), "mv_quantize_into_stack")


def int8_expert_loaders(blocks: dict):
    """Loader hooks {checkpoint key: fn(tensor)} for the routed experts of each named block, as
    engine.py:_int8_expert_loaders builds them: `<name>.experts.<e>.gate_proj.weight` -> q_gu rows [0, I) of slot
    e, `up_proj` -> rows [I, 2I), `down_proj` -> q_d slot e. `blocks` maps a module name to
    (q_gu, s_gu, q_d, s_d, n_experts)."""
    hooks = {}
    for name, (q_gu, s_gu, q_d, s_d, n_experts) in blocks.items():
        I = q_gu.shape[1] // 2
        for e in range(n_experts):
            p = f"{name}.experts.{e}."
            hooks[p + "gate_proj.weight"] = lambda src, e=e, q=q_gu, s=s_gu: quantize_into(q, s, e, 0, src)
            hooks[p + "up_proj.weight"] = lambda src, e=e, q=q_gu, s=s_gu, I=I: quantize_into(q, s, e, I, src)
            hooks[p + "down_proj.weight"] = lambda src, e=e, q=q_d, s=s_d: quantize_into(q, s, e, 0, src)
    return hooks


def run_hooks(tensors: dict, hooks: dict, device, workers: int = 4):
    """Feed checkpoint tensors {key: tensor} to their hooks from `workers` threads, each on its own CUDA stream
    (the loader's threading, direct_load.py:109-135); returns the keys handled. Waits for every stream."""
    items = [(k, t) for k, t in tensors.items() if k in hooks]
    groups = [items[i::workers] for i in range(workers)]
    dev = torch.device(device)

    def work(group):
        stream = torch.cuda.Stream(device=dev)
        with torch.cuda.stream(stream):
            for k, t in group:
                hooks[k](t)
        stream.synchronize()
        return [k for k, _ in group]

    with ThreadPoolExecutor(workers) as ex:
        done = [k for ks in ex.map(work, groups) for k in ks]
    return done
