"""The C ABI library loads and exports every symbol include/i4d.h declares."""
import ctypes
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared():
    text = open(os.path.join(ROOT, "include", "i4d.h")).read()
    return sorted(set(re.findall(r"\b(i4d_[a-z0-9_]+)\s*\(", text)))


def test_header_matches_shim_list(pkg):
    assert _declared() == sorted(pkg.EXPORTS)


def test_library_exports_all_symbols(pkg):
    lib = ctypes.CDLL(pkg.LIB_PATH)
    for name in _declared():
        assert hasattr(lib, name), name


def test_library_is_sm100a_cuda_build(pkg):
    # The product library carries device code; no CPU implementation exists.
    data = open(pkg.LIB_PATH, "rb").read()
    assert b"sm_100a" in data or b"sm_100" in data
