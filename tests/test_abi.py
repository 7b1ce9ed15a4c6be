"""The C ABI library loads and exports every symbol include/i4d.h declares;
on a GPU, the loaded device code reports the sm_100a build target."""
import ctypes
import os
import re

import pytest

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


@pytest.mark.gpu
def test_library_runs_sm100a_device_code(pkg):
    # The token kernel's binary version, queried from the CUDA runtime: the
    # library carries sm_100a code and no CPU implementation.
    binary, cc = pkg.device_arch(0)
    assert binary == 100, binary
    assert cc == 100, cc
