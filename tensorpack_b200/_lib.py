"""ctypes binding of the native library (include/mtc_b200.h).

Loading never falls back to anything else: a missing or unloadable
``libmtc_b200.so`` raises ``NativeLibraryError`` at the first call that
needs the GPU path.
"""

from __future__ import annotations

import ctypes
import os
import threading

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "libmtc_b200.so")

MTC_OK = 0
MTC_ERR_INVALID = -1
MTC_ERR_CUDA = -2
MTC_ERR_WORKSPACE = -3
MTC_ERR_UNSUPPORTED = -4

STATUS_TIMEOUT = 1
STATUS_X_RANGE = 2
STATUS_BAD_STREAM = 4

c_u8, c_u16, c_u32, c_u64 = ctypes.c_uint8, ctypes.c_uint16, ctypes.c_uint32, ctypes.c_uint64
c_i32, c_i64, c_p, c_size = ctypes.c_int32, ctypes.c_int64, ctypes.c_void_p, ctypes.c_size_t


class NativeLibraryError(RuntimeError):
    """The CUDA library is missing or failed to load."""


class StreamDesc(ctypes.Structure):
    """struct mtc_stream_desc."""

    _fields_ = [
        ("records", c_p), ("tiles", c_p), ("row_off", c_p),
        ("K", c_i32), ("N", c_i32), ("tk", c_i32), ("tn", c_i32),
        ("band_tiles", c_i32), ("exp2", c_i32),
        ("record_bytes", c_u64), ("max_row_bytes", c_u32), ("scale_words", c_i32),
        ("stage_images", c_p), ("stage_counts", c_p), ("stage_offsets", c_p), ("stage_ranges", c_p),
        ("max_stage_bytes", c_u32), ("max_sms", c_u32),
    ]


assert ctypes.sizeof(StreamDesc) == 104


class StripDesc(ctypes.Structure):
    """struct mtc_strip_desc (all pointers on the device)."""

    _fields_ = [
        ("stream", c_p), ("batch_off", c_p), ("strip_batch", c_p),
        ("work", c_p), ("warp_work", c_p), ("red", c_p), ("cta_red", c_p),
        ("K", c_i32), ("N", c_i32), ("tk", c_i32), ("tn", c_i32),
        ("n_strips", c_i32), ("n_batches", c_i32), ("exp2", c_i32), ("max_batch_bytes", c_u32),
        ("n_cta", c_i32), ("n_warps", c_i32), ("max_cta_slots", c_u32), ("flags", c_u32), ("stream_bytes", c_u64),
    ]


assert ctypes.sizeof(StripDesc) == 112
STRIP_WIDE = 1
STRIP_MERGE_MODES = 2


class Epilogue(ctypes.Structure):
    """struct mtc_epilogue: Y = act(acc + bias[col])."""

    _fields_ = [("bias", c_p), ("act", c_i32), ("pad_", c_i32)]


assert ctypes.sizeof(Epilogue) == 16
ACT_NONE, ACT_RELU, ACT_SILU, ACT_GELU_TANH = 0, 1, 2, 3
ACTIVATIONS = {None: ACT_NONE, "none": ACT_NONE, "relu": ACT_RELU, "silu": ACT_SILU, "gelu_tanh": ACT_GELU_TANH}
_EP = ctypes.POINTER(Epilogue)

# name -> (restype, argtypes); every symbol declared in include/mtc_b200.h.
SIGNATURES = {
    "mtc_abi_version": (c_i32, []),
    "mtc_last_error": (ctypes.c_char_p, []),
    "mtc_device_sm_count": (c_i32, [c_i32]),
    "mtc_copy_async": (c_i32, [c_p, c_p, c_size, c_p]),
    "mtc_set_wait_limit_ns": (c_i32, [c_u64]),
    "mtc_debug_withhold_bytes": (c_i32, [c_u32]),
    "mtc_repack_plan": (c_i32, [c_p, c_p, c_i32, c_i32, c_i32, c_i32, c_p, c_p, c_p,
                                ctypes.POINTER(c_u64), c_p]),
    "mtc_repack_fill": (c_i32, [c_p, c_u64, c_p, c_p, ctypes.POINTER(StreamDesc), c_p, c_p, c_p]),
    "mtc_repack_stage_plan": (c_i32, [ctypes.POINTER(StreamDesc), c_p, c_p, c_p, c_p, ctypes.POINTER(c_u64), c_p]),
    "mtc_repack_stage_fill": (c_i32, [ctypes.POINTER(StreamDesc), c_p, c_p, c_p]),
    "mtc_rd_search": (c_i32, [c_p, c_i32, c_i32, c_i32, c_p, c_i32, c_p, c_i32, c_i32, c_p, c_p, c_p]),
    "mtc_dequant": (c_i32, [ctypes.POINTER(StreamDesc), c_p, c_p, c_p, c_i64, c_p]),
    "mtc_gemv_workspace_bytes": (c_size, [ctypes.POINTER(StreamDesc), c_i32, c_i32]),
    "mtc_gemv": (c_i32, [ctypes.POINTER(StreamDesc), c_p, c_i32, c_i64, c_p, c_p, c_p, c_i64, c_i32,
                         c_p, c_size, c_p, c_p, c_p]),
    "mtc_gemv_static": (c_i32, [ctypes.POINTER(StreamDesc), c_p, c_i32, c_i64, c_p, c_p, c_p, c_i64, c_p, c_p]),
    "mtc_decode_workspace_bytes": (c_size, [ctypes.POINTER(StreamDesc), c_i32]),
    "mtc_decode": (c_i32, [ctypes.POINTER(StreamDesc), c_p, c_i32, c_i64, c_p, c_p, c_p, c_i64, c_p, c_size, c_p,
                           c_p, _EP, c_p]),
    "mtc_strip_plan": (c_i32, [c_p, c_p, c_i32, c_i32, c_i32, c_u32, c_u32, c_u32, ctypes.POINTER(c_u64)]),
    "mtc_strip_fill": (c_i32, [c_p, c_u64, c_p, c_p, c_i32, c_i32, c_i32, c_u32, c_u32, c_u32, c_p, c_p, c_p]),
    "mtc_strip_check": (c_i32, [c_p, c_u64, c_p, c_p, c_i32, c_i32, c_i32, c_u32, c_u32]),
    "mtc_strip_schedule": (c_i32, [c_p, c_p, c_p, c_i32, c_i32, c_i32, c_u32, c_p, c_p, c_p, c_p,
                                   ctypes.POINTER(c_u32)]),
    "mtc_strip_fits": (c_i32, [ctypes.POINTER(StripDesc), c_i32]),
    "mtc_strip_decode": (c_i32, [ctypes.POINTER(StripDesc), c_p, c_i32, c_i64, c_p, c_p, c_p, c_i64, c_p, _EP, c_p]),
    "mtc_prefill_workspace_bytes": (c_size, [ctypes.POINTER(StreamDesc), c_i32, c_i32]),
    "mtc_gemm_prefill": (c_i32, [ctypes.POINTER(StreamDesc), c_p, c_i32, c_i64, c_p, c_p, c_p, c_i64,
                                 c_p, c_size, c_p, _EP, c_p]),
    "mtc_prefill_gather": (c_i32, [ctypes.POINTER(StreamDesc), c_p, c_i32, c_i64, c_p, c_p, c_size, c_p, c_p]),
    "mtc_prefill_gemm": (c_i32, [ctypes.POINTER(StreamDesc), c_i32, c_p, c_i64, c_i32, c_p, c_size, c_p, _EP,
                                 c_p]),
    "mtc_prefill_scatter": (c_i32, [ctypes.POINTER(StreamDesc), c_i32, c_p, c_p, c_i64, c_p, c_size, _EP, c_p]),
    "mtc_permute_rows": (c_i32, [c_p, c_i64, c_i64, c_i32, c_i32, c_p, c_i32, c_i32, c_p, c_i64, _EP, c_p]),
}

_lock = threading.Lock()
_lib = None


def load(path: str = LIB_PATH):
    """Load (once) and return the ctypes library with prototypes attached."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(path):
            raise NativeLibraryError(
                f"{path} not found: build it with `python -m tensorpack_b200.build` (nvcc, sm_100a)")
        try:
            lib = ctypes.CDLL(path)
        except OSError as e:
            raise NativeLibraryError(f"cannot load {path}: {e}") from e
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        if lib.mtc_abi_version() != 2:
            raise NativeLibraryError("libmtc_b200.so ABI version mismatch")
        _lib = lib
        return lib


def check(rc: int, what: str):
    """Map a C return code to the reference's Python exception types."""
    if rc == MTC_OK:
        return
    msg = (load().mtc_last_error() or b"").decode(errors="replace")
    text = f"{what}: {msg or 'error ' + str(rc)}"
    if rc in (MTC_ERR_INVALID, MTC_ERR_WORKSPACE):
        raise ValueError(text)
    if rc == MTC_ERR_UNSUPPORTED:
        raise NotImplementedError(text)
    raise RuntimeError(text)
