"""Host side of the strip stream, the decode-sized (M <= 4) device layout.

The stream is built on the host by the native library (``mtc_strip_plan`` /
``mtc_strip_fill``, pure host code in csrc/mtc_strip_build.cu) from the same
leaf list and reference-layout arena the GPU repack reads
(mtc/kernels/gemm.py:449-478), then uploaded by ``DeviceStream``.  A strip is
8 output features over all of K; its 8x8 groups and 4x4 micro-blocks are
sorted by precision into steps of straight-line decode, and the steps of a
strip are grouped into batch records of at most ``batch_bytes`` bytes that
the kernel moves with one bulk copy each.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass
from math import ceil, log2

import numpy as np

from .. import _lib
from . import layout

# Version of the strip stream layout (step records, descriptors, batch
# records).  A stream saved by another version is rebuilt on load.
STRIP_FORMAT_VERSION = 1
BATCH_BYTES = 4096   # largest batch record (one shared-memory slot of the kernel)
BATCH_STEPS = 64     # most steps per batch record
MAX_M = 4            # tokens per strip-kernel call
WARPS = 16           # warps per CTA of the decode kernel's schedule (M = 2..4)
WARPS_M1 = 24        # ... and for M = 1 (fewer registers per token: more warps fit)


def strip_exp2(ls: layout.LeafSet) -> int:
    """Power-of-two pre-scale of the stream's scales: the largest |scale| of
    a live leaf maps to at most 1, so |x * scale| stays within the checked
    fp16 range of x."""
    live = (ls.mode != 0) & (ls.scale != 0)
    if not live.any():
        return 0
    smax = float(np.max(np.abs(ls.scale[live].astype(np.float64))))
    if not np.isfinite(smax) or smax <= 0.0:
        return 0
    return int(max(-100, min(100, -ceil(log2(smax)))))


@dataclass
class HostStripStream:
    """A strip stream in host memory (numpy arrays) with its geometry."""

    K: int
    N: int
    tk: int
    tn: int
    exp2: int
    stream: np.ndarray       # uint8, batch records
    batch_off: np.ndarray    # uint32 [n_batches + 1]
    strip_batch: np.ndarray  # uint32 [n_strips + 1]
    max_batch_bytes: int
    flags: int = 0           # 0 or _lib.STRIP_WIDE

    @property
    def n_strips(self) -> int:
        return int(self.strip_batch.shape[0] - 1)

    @property
    def n_batches(self) -> int:
        return int(self.batch_off.shape[0] - 1)

    def schedule(self, n_cta: int, n_warps: int = WARPS) -> "StripSchedule":
        """The decode kernel's static schedule on ``n_cta`` CTAs (capped at the
        strip count) of ``n_warps`` warps, built on the host."""
        lib = _lib.load()
        n_cta = max(1, min(int(n_cta), self.n_strips))
        work = np.zeros(2 * self.n_batches, dtype=np.uint32)
        warp_work = np.zeros(n_cta * n_warps + 1, dtype=np.uint32)
        red = np.zeros(3 * self.n_strips, dtype=np.uint32)
        cta_red = np.zeros(n_cta + 1, dtype=np.uint32)
        slots = ctypes.c_uint32()
        _lib.check(lib.mtc_strip_schedule(self.stream.ctypes.data, self.batch_off.ctypes.data,
                                          self.strip_batch.ctypes.data, self.n_strips, n_cta, int(n_warps),
                                          int(self.flags), work.ctypes.data, warp_work.ctypes.data, red.ctypes.data,
                                          cta_red.ctypes.data, ctypes.byref(slots)), "strip schedule")
        return StripSchedule(n_cta, int(n_warps), work, warp_work, red, cta_red, slots.value)

    def desc(self, stream_ptr, batch_off_ptr, strip_batch_ptr, sched: "StripSchedule", sched_ptrs) -> _lib.StripDesc:
        """The C descriptor with the device pointers of an uploaded copy of
        the stream and of ``sched``'s arrays (work, warp_work, red, cta_red)."""
        work, warp_work, red, cta_red = sched_ptrs
        return _lib.StripDesc(
            stream=stream_ptr, batch_off=batch_off_ptr, strip_batch=strip_batch_ptr, work=work, warp_work=warp_work,
            red=red, cta_red=cta_red, K=self.K, N=self.N, tk=self.tk, tn=self.tn, n_strips=self.n_strips,
            n_batches=self.n_batches, exp2=self.exp2, max_batch_bytes=self.max_batch_bytes, n_cta=sched.n_cta,
            n_warps=sched.n_warps, max_cta_slots=sched.max_slots, flags=self.flags,
            stream_bytes=int(self.stream.nbytes))


@dataclass
class StripSchedule:
    """Static schedule of the strip decode kernel (mtc_strip_schedule): work
    items {offset, (bytes / 16) | slot << 12 | flush << 31} in warp order,
    the first item of each warp, and per CTA the strips with their
    partial-sum slot ranges."""

    n_cta: int
    n_warps: int
    work: np.ndarray       # uint32 [2 n_batches]
    warp_work: np.ndarray  # uint32 [n_cta n_warps + 1]
    red: np.ndarray        # uint32 [3 n_strips]
    cta_red: np.ndarray    # uint32 [n_cta + 1]
    max_slots: int


def build_host(mat, batch_bytes: int = BATCH_BYTES, batch_steps: int = BATCH_STEPS,
               wide: bool = False, merge_modes: bool = True) -> HostStripStream:
    """Build the strip stream of an MTCMatrix on the host (no GPU needed).
    ``wide`` packs group steps of 16 groups with two micro-blocks per lane
    (MTC_STRIP_WIDE, measured slower on the B200, kept for comparison);
    ``merge_modes`` (default) packs P2 items with the P3 decoder and P6 items
    with the P8 one: exact, and fewer step kinds and partial steps."""
    flags = (_lib.STRIP_WIDE if wide else 0) | (_lib.STRIP_MERGE_MODES if merge_modes else 0)
    lib = _lib.load()
    K, N = (int(v) for v in mat.shape)
    ls = mat.leaf_set
    leaves, begin, tk, tn = layout.device_leaf_list(ls, K, N)
    exp2 = strip_exp2(ls)
    arena = np.ascontiguousarray(mat.arena.raw_buffer[:max(mat.total_bytes_allocated, 1)])
    leaves = np.ascontiguousarray(leaves)
    begin = np.ascontiguousarray(begin, dtype=np.uint32)
    out = (ctypes.c_uint64 * 4)()
    _lib.check(lib.mtc_strip_plan(leaves.ctypes.data, begin.ctypes.data, tk, tn, exp2, batch_bytes, batch_steps,
                                  flags, out), "strip plan")
    total, n_batches, n_strips, max_batch = (int(v) for v in out)
    # 16 spare bytes so that every record can be read with 16-byte loads
    stream = np.zeros(total + 16, dtype=np.uint8)
    batch_off = np.zeros(n_batches + 1, dtype=np.uint32)
    strip_batch = np.zeros(n_strips + 1, dtype=np.uint32)
    _lib.check(lib.mtc_strip_fill(arena.ctypes.data, arena.nbytes, leaves.ctypes.data, begin.ctypes.data, tk, tn,
                                  exp2, batch_bytes, batch_steps, flags, stream.ctypes.data, batch_off.ctypes.data,
                                  strip_batch.ctypes.data), "strip fill")
    hs = HostStripStream(K, N, tk, tn, exp2, stream, batch_off, strip_batch, max_batch, flags & _lib.STRIP_WIDE)
    check(hs)
    return hs


def check(hs: HostStripStream) -> None:
    """Validate every record of a host strip stream (raises ValueError)."""
    lib = _lib.load()
    _lib.check(lib.mtc_strip_check(hs.stream.ctypes.data, hs.stream.nbytes, hs.batch_off.ctypes.data,
                                   hs.strip_batch.ctypes.data, hs.n_batches, hs.n_strips, hs.tk,
                                   hs.max_batch_bytes, hs.flags), "strip stream")


def export_host(hs: HostStripStream) -> tuple:
    """(metadata, name -> array) of a host strip stream, for the on-disk
    format (tensorpack_b200.core.fileformat)."""
    meta = {"version": STRIP_FORMAT_VERSION, "K": hs.K, "N": hs.N, "tk": hs.tk, "tn": hs.tn, "exp2": hs.exp2,
            "flags": int(hs.flags), "max_batch_bytes": int(hs.max_batch_bytes)}
    return meta, {"stream": hs.stream, "batch_off": hs.batch_off, "strip_batch": hs.strip_batch}


def import_host(mat, meta: dict, arrs: dict) -> "HostStripStream | None":
    """A saved strip stream for ``mat``, validated record by record, or None
    when it was written by another layout version or for another matrix
    (the caller then builds it again).  Raises ValueError on a stream that
    claims this version but fails validation."""
    K, N = (int(v) for v in mat.shape)
    try:
        ok = (int(meta["version"]) == STRIP_FORMAT_VERSION and int(meta["K"]) == K and int(meta["N"]) == N
              and int(meta["tk"]) == -(-K // layout.TILE) and int(meta["tn"]) == -(-N // layout.TILE)
              and int(meta["exp2"]) == strip_exp2(mat.leaf_set)
              # only the default form is attached to a matrix; another form
              # (wide steps, larger batch records) is rebuilt in the default one
              and int(meta.get("flags", 0)) == 0 and int(meta.get("max_batch_bytes", 0)) <= BATCH_BYTES)
    except (KeyError, TypeError, ValueError):
        return None
    if not ok:
        return None
    try:
        stream = np.ascontiguousarray(arrs["stream"], dtype=np.uint8)
        batch_off = np.ascontiguousarray(arrs["batch_off"], dtype=np.uint32)
        strip_batch = np.ascontiguousarray(arrs["strip_batch"], dtype=np.uint32)
        hs = HostStripStream(K, N, int(meta["tk"]), int(meta["tn"]), int(meta["exp2"]), stream, batch_off,
                             strip_batch, int(meta["max_batch_bytes"]), int(meta["flags"]))
    except (KeyError, TypeError, ValueError) as e:
        raise ValueError(f"saved strip stream: {e}") from None
    if hs.n_strips != 4 * hs.tn or hs.n_batches < hs.n_strips:
        raise ValueError("saved strip stream: table sizes do not match the matrix")
    check(hs)
    return hs