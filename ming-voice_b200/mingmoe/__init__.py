"""mingmoe: host side of the B200 (sm_100a) MoE block kernels for ming-voice.

The compute path is the C-ABI library libmingmoe.so (include/mingmoe.h); this package marshals torch tensors
into it. There is no CPU fallback: calls on CPU tensors, or without the built library, raise."""
from . import _lib  # noqa: F401

__version__ = "0.1.0"
