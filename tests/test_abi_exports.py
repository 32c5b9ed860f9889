"""The C-ABI library builds for sm_100a, loads without a GPU and exports
every entry point declared in include/mtc_b200.h (no compute calls here)."""

import ctypes
import os
import re

import pytest

from tensorpack_b200 import _lib, build

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    text = open(os.path.join(ROOT, "include", "mtc_b200.h")).read()
    return sorted(set(re.findall(r"^MTC_API\s+[\w\s\*]+?\b(mtc_\w+)\s*\(", text, flags=re.M)))


@pytest.fixture(scope="module")
def lib():
    build.build()
    return _lib.load()


def test_header_declares_entry_points():
    names = declared_symbols()
    assert {"mtc_repack_plan", "mtc_repack_fill", "mtc_dequant", "mtc_gemv"} <= set(names)


def test_every_declared_symbol_is_exported(lib):
    for name in declared_symbols():
        assert hasattr(lib, name), name
        assert name in _lib.SIGNATURES, f"{name} has no ctypes prototype"


def test_abi_version_and_error_text(lib):
    assert lib.mtc_abi_version() == 2
    assert isinstance(lib.mtc_last_error(), bytes)


def test_struct_sizes_match_header():
    assert ctypes.sizeof(_lib.StreamDesc) == 104
    from tensorpack_b200.core.layout import LEAF_IN_DTYPE
    assert LEAF_IN_DTYPE.itemsize == 12


def test_invalid_arguments_fail_without_gpu(lib):
    """Argument validation happens before any CUDA call."""
    rc = lib.mtc_gemv(None, None, 1, 1, None, None, None, 1, 0, None, 0, None, None, None)
    assert rc == _lib.MTC_ERR_INVALID
    assert b"null" in lib.mtc_last_error()
