"""ctypes binding of the C-ABI library `libmingmoe.so` (declared in include/mingmoe.h).

The library is the only compute path: there is no CPU or PyTorch fallback. Loading fails with an
ImportError naming the build command when the library is missing, and every entry point raises
RuntimeError with the library's message when it returns a non-zero status.
"""
from __future__ import annotations

import ctypes as C
import os
import threading

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("MINGMOE_LIB", os.path.join(HERE, "libmingmoe.so"))

MV_OK, MV_ERR_INVALID, MV_ERR_ALIGN, MV_ERR_CUDA, MV_ERR_UNSUPPORTED, MV_ERR_WORKSPACE = range(6)
MV_BF16, MV_F16, MV_F32, MV_I8, MV_I32, MV_I64 = range(6)
MV_ROUTE_SOFTMAX, MV_ROUTE_SIGMOID_GROUP = 0, 1

_DT = {torch.bfloat16: MV_BF16, torch.float16: MV_F16, torch.float32: MV_F32, torch.int8: MV_I8,
       torch.int32: MV_I32, torch.int64: MV_I64}

P = C.c_void_p
I32 = C.c_int
I64 = C.c_longlong
SZ = C.c_size_t
F32 = C.c_float
F64 = C.c_double


class MoeWeights(C.Structure):
    """mirror of `mv_moe_weights`"""
    _fields_ = [("w_gu", P), ("w_d", P), ("s_gu", P), ("s_d", P), ("w_dtype", I32), ("s_dtype", I32),
                ("E1", I32), ("H", I32), ("I", I32), ("pad0", I32), ("gu_se", I64), ("gu_sr", I64),
                ("d_se", I64), ("d_sr", I64), ("sgu_se", I64), ("sd_se", I64)]


class Block(C.Structure):
    """mirror of `mv_block`"""
    _fields_ = [("experts", MoeWeights), ("norm_w", P), ("router_w", P), ("router_scale", P), ("router_bias", P),
                ("eps", F32), ("router_dtype", I32), ("router_scale_dtype", I32), ("E", I32), ("top_k", I32),
                ("route_mode", I32), ("n_group", I32), ("topk_group", I32), ("n_shared", I32), ("shared_id", I32),
                ("residual_from_x", I32), ("pad0", I32), ("route_scale", F64), ("next", P)]


_SIGS = {
    "mv_version": (I32, []),
    "mv_last_error": (C.c_char_p, []),
    "mv_workspace_status": (I32, [P, I32, C.POINTER(C.c_uint), C.POINTER(C.c_uint), P]),
    "mv_rmsnorm": (I32, [P, I32, I64, P, I32, P, I32, I32, I32, F32, P]),
    "mv_route": (I32, [I32, P, I64, P, I32, P, I32, P, I32, I32, I32, I32, I32, I32, F64, I32, I32, P, P, I32, P,
                       P, SZ, P]),
    "mv_route_workspace_bytes": (SZ, [I32, I32]),
    "mv_quantize_rows_int8": (I32, [P, I32, I64, I64, I32, P, P, I32, P]),
    "mv_dequant_rows_int8": (I32, [P, P, I32, I64, I32, P, P]),
    "mv_moe_decode": (I32, [C.POINTER(MoeWeights), P, I64, P, F32, P, I32, P, I32, I32, P, P, P, SZ, P]),
    "mv_moe_decode_workspace_bytes": (SZ, [I32, I32, I32, I32]),
    "mv_block_decode": (I32, [C.POINTER(Block), P, I32, P, P, P, I32, P, P, SZ, P]),
    "mv_block_decode_workspace_bytes": (SZ, [I32, I32, I32, I32]),
    "mv_block_decode_workspace_bytes_tc": (SZ, [C.POINTER(Block), I32]),
    "mv_moe_decode_workspace_bytes_tc": (SZ, [I32, I32, I32, I32, I32]),
    "mv_block_decode_noalloc": (I32, [C.POINTER(Block), P, I32, P, P, P, I32, P, P, P]),
    "mv_moe_align": (I32, [P, I32, I32, I32, I32, P, P, P, P, SZ, P]),
    "mv_small_linear": (I32, [P, I64, P, I64, P, P, I64, P, F32, I32, P, I64, I32, I32, I32, P]),
    "mv_moe_align_workspace_bytes": (SZ, [I32, I32]),
    "mv_moe_prefill": (I32, [C.POINTER(MoeWeights), P, I64, P, I32, P, I32, I32, P, I64, P, P, SZ, P]),
    "mv_moe_prefill_workspace_bytes": (SZ, [I32, I32, I32, I32, I32, I32]),
    "mv_quantize_into_stack": (I32, [P, I32, I64, I32, I32, P, P, I32, I32, I32, I32, I32, P]),
    "mv_mask_pad_rows": (I32, [P, I32, I32, I32, P, P]),
    "mv_moe_prefill_f32": (I32, [C.POINTER(MoeWeights), P, I64, I32, P, I64, P, I32, P, I32, I32, P, I64, P, I32, P,
                                 SZ, P]),
    "mv_ep_workspace_bytes": (SZ, []),
    "mv_ep_plan": (I32, [P, P, I32, I32, I32, P, P, I32, I32, I32, I32, P, P, P, P, P, P, SZ, P]),
    "mv_ep_pack": (I32, [P, I64, I32, P, P, I32, I32, P, P]),
    "mv_ep_unpack": (I32, [P, I32, I32, I32, I32, P, P, P]),
    "mv_ep_narrow": (I32, [P, I64, P, P]),
    "mv_ep_combine": (I32, [P, I64, P, P, I32, P, I32, I32, I32, P, P]),
}

_lib = None
_lock = threading.Lock()


def lib():
    """Load the library once (raises ImportError if it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise ImportError(f"{LIB_PATH} is missing: build it with `python ming-voice_b200/mingmoe/build.py` "
                                  "(or __graft_entry__.build())")
            L = C.CDLL(LIB_PATH)
            for name, (res, args) in _SIGS.items():
                if hasattr(L, name):
                    f = getattr(L, name)
                    f.restype = res
                    f.argtypes = args
            _lib = L
    return _lib


def exported_symbols():
    return list(_SIGS)


def check(rc: int, what: str):
    if rc != MV_OK:
        msg = lib().mv_last_error().decode(errors="replace")
        raise RuntimeError(f"{what} failed (status {rc}): {msg}")


def dt(t_or_dtype) -> int:
    d = t_or_dtype.dtype if isinstance(t_or_dtype, torch.Tensor) else t_or_dtype
    if d not in _DT:
        raise TypeError(f"unsupported dtype {d}")
    return _DT[d]


def ptr(t):
    return None if t is None else C.c_void_p(t.data_ptr())


def stream_ptr(device=None):
    return C.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def require_cuda(*tensors):
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise RuntimeError("mingmoe kernels run on the GPU only: got a CPU tensor")


# ---------------------------------------------------------------------------------------------- workspaces

_ws: dict = {}
# Workspaces replaced by a larger one. A CUDA graph captured while one of them was current keeps its address
# and writes to it on every replay, so a superseded buffer is never returned to the allocator: it stays alive
# (and is still checked by all_workspace_errors) for the life of the process.
_retired: list = []


def workspace(kind: str, nbytes: int, device: torch.device) -> torch.Tensor:
    """A zero-initialised uint8 device buffer of >= nbytes reused by every call of `kind` on the current
    stream (the kernels leave it zeroed). Creating or growing one is not allowed during stream capture; a buffer
    outgrown by a later eager call is kept alive, not freed, because a captured graph may still use it."""
    stream = torch.cuda.current_stream(device)
    key = (kind, device.index if device.index is not None else torch.cuda.current_device(), stream.cuda_stream)
    buf = _ws.get(key)
    if buf is None or buf.numel() < nbytes:
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError(f"mingmoe workspace '{kind}' ({nbytes} bytes) must be created before graph capture; "
                               "run the call once eagerly first")
        nb = max(nbytes, 1 << 16)
        if buf is not None:
            nb = max(nb, 2 * buf.numel())  # geometric growth: few superseded buffers stay alive
            _retired.append((key, buf))
        buf = torch.zeros(nb, dtype=torch.uint8, device=device)
        _ws[key] = buf
    return buf


def workspace_status(buf: torch.Tensor, clear=True):
    code, info = C.c_uint(0), C.c_uint(0)
    check(lib().mv_workspace_status(ptr(buf), int(clear), C.byref(code), C.byref(info), stream_ptr(buf.device)),
          "mv_workspace_status")
    return code.value, info.value


def all_workspace_errors(clear=True):
    """Device-side error words of every cached workspace: {(kind, device, stream): (code, info)} for non-zero."""
    out = {}
    for k, buf in list(_ws.items()) + [((*k, "retired", n), b) for n, (k, b) in enumerate(_retired)]:
        c, i = workspace_status(buf, clear)
        if c:
            out[k] = (c, i)
    return out
