"""CPU checks of the C-ABI library: it loads without a GPU and exports every symbol include/mingmoe.h declares,
the ctypes prototypes match the header, and the host-side argument checks reject bad calls before any
kernel launch."""
import os
import re

import pytest
import torch

from conftest import ROOT
from mingmoe import _lib as L


def header_symbols():
    src = open(os.path.join(ROOT, "include", "mingmoe.h")).read()
    return sorted(set(re.findall(r"^MV_API\s+[\w\s\*]+?\b(mv_\w+)\s*\(", src, flags=re.M)))


def test_header_symbols_exported():
    lib = L.lib()
    syms = header_symbols()
    assert len(syms) >= 10
    for s in syms:
        assert hasattr(lib, s), s
    # every declared symbol has a ctypes prototype
    assert set(syms) <= set(L.exported_symbols()), set(syms) - set(L.exported_symbols())


def test_version_and_error_string():
    assert L.lib().mv_version() >= 100
    assert isinstance(L.lib().mv_last_error(), bytes)


def test_argument_checks_run_on_host():
    lib = L.lib()
    # null pointers and bad sizes fail before touching the device
    assert lib.mv_rmsnorm(None, 0, 0, None, 0, None, 0, 1, 16, 1e-6, None) == L.MV_ERR_INVALID
    assert b"null" in lib.mv_last_error()
    w = L.MoeWeights()
    assert lib.mv_moe_decode(None, None, 0, None, 0.0, None, 0, None, 1, 1, None, None, None, 0, None) == L.MV_ERR_INVALID
    assert lib.mv_route(7, None, 0, None, 0, None, 0, None, 1, 16, 8, 2, 1, 1, 1.0, 0, 0, None, None, 4, None, None,
                        0, None) == L.MV_ERR_INVALID
    del w


def test_cpu_tensors_rejected():
    import fused_ops
    with pytest.raises(RuntimeError):
        fused_ops.rms_norm(torch.ones(2, 8), torch.ones(8), 1e-6)
