"""The C-ABI library loads and exports every symbol include/umsx.h declares (CPU only)."""
import ctypes
import os
import re

from tests.helpers import U

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    text = open(os.path.join(ROOT, "include", "umsx.h")).read()
    return sorted(set(re.findall(r"\b(umsx_[a-z0-9_]+)\s*\(", text)))


def test_header_matches_binding_list():
    assert declared_symbols() == sorted(U.EXPORTS)


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(U.LIB_PATH)
    for name in declared_symbols():
        assert hasattr(lib, name), name
    assert U.lib().umsx_version() == 1


def test_errors_without_a_device_are_statuses_not_crashes():
    """Invalid descriptors are rejected before any device call."""
    d = U.Desc(100, 64, 8, 2, U.QUANT_MXFP4, 0, 1, 1, 0, 0, 1.702, 7.0, 1.0, 4, 0, 1)
    h = ctypes.c_void_p()
    st = U.lib().umsx_moe_create_synthetic(ctypes.byref(d), 0, 0, 0.02, 0.1, 0.02, 0, 0, ctypes.byref(h))
    assert st == U.EINVAL and b"multiples of 64" in U.lib().umsx_last_error()
