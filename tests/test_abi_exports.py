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


def test_library_records_its_source_hash(lib):
    """The built library carries the hash of the sources it was built from,
    so a stale prebuilt library next to changed sources is rebuilt."""
    assert build.library_hash() == build.source_hash()
    assert not build.needs_build()


def test_wait_limit_and_hold_arguments(lib):
    """The timeout diagnostics validate their arguments without a GPU."""
    assert lib.mtc_debug_withhold_bytes(8) == _lib.MTC_ERR_INVALID
    assert lib.mtc_debug_withhold_bytes(8192) == _lib.MTC_ERR_INVALID
    assert lib.mtc_debug_withhold_bytes(0) == 0
    assert lib.mtc_set_wait_limit_ns(0) == 0
