"""Device-resident tile stream of a packed MTC matrix and the kernel launchers.

``DeviceStream`` owns the GPU copy of one matrix (tile records, 16-byte tile
descriptors, per-band row offsets, permutations) as torch tensors and calls
the C ABI with their device pointers on the current torch stream.  torch is
only the allocator / stream provider here; every byte of the stream is
produced and consumed by the CUDA kernels in ``csrc/``.
"""

from __future__ import annotations

import ctypes
from typing import Optional

import numpy as np
import torch

from .. import _lib
from ..core import layout

BAND_TILES = 8  # tiles per column band = 256 output features (one per consumer warp)
DECODE_MAX_M = 16  # largest M served by the split-K decode kernel
STRIP_MAX_M = 4    # largest M served by the strip-stream decode kernel
# Version of the device tile stream layout (tile descriptors, records, row
# offsets, sub-stage images).  A stream saved by another version is rebuilt
# from the host layout instead of uploaded.
STREAM_FORMAT_VERSION = 4
_STREAM_ARRAYS = ("tiles", "row_off", "records", "stage_counts", "stage_offsets", "stage_ranges", "stage_images")


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def epilogue(bias: Optional[torch.Tensor] = None, activation=None) -> Optional[_lib.Epilogue]:
    """The fused output epilogue Y = act(acc + bias[col]) of the kernels, or
    None for a plain product.  ``bias`` is a contiguous fp32 CUDA tensor with
    one value per output column of Y as written; ``activation`` is None,
    "relu", "silu" or "gelu_tanh".  The caller keeps ``bias`` alive until
    the kernel has run (the returned struct holds its device pointer)."""
    if activation not in _lib.ACTIVATIONS:
        raise ValueError(f"unknown activation {activation!r} (one of relu, silu, gelu_tanh)")
    act = _lib.ACTIVATIONS[activation]
    if bias is None and act == _lib.ACT_NONE:
        return None
    if bias is not None:
        if bias.dtype != torch.float32 or not bias.is_cuda or not bias.is_contiguous() or bias.dim() != 1:
            raise ValueError("bias must be a contiguous 1-D float32 CUDA tensor")
    return _lib.Epilogue(bias=None if bias is None else bias.data_ptr(), act=act)


def _ep(e: Optional[_lib.Epilogue]):
    return None if e is None else ctypes.byref(e)


def stream_compatible(meta: dict, mat) -> bool:
    """Whether a saved stream was made by this device format for ``mat``."""
    K, N = mat.shape
    try:
        return (int(meta["version"]) == STREAM_FORMAT_VERSION and int(meta["band_tiles"]) == BAND_TILES
                and int(meta["K"]) == K and int(meta["N"]) == N and int(meta["tk"]) == -(-K // layout.TILE)
                and int(meta["tn"]) == -(-N // layout.TILE) and int(meta["exp2"]) == layout.choose_exp2(mat.leaf_set)
                and int(meta["scale_words"]) == (1 if layout.bf16_exact(np.asarray(mat.scales)) else 2))
    except (KeyError, TypeError, ValueError):
        return False


def check_stream_buffers(meta: dict, arrs: dict) -> None:
    """Host-side consistency checks of a saved stream before it is uploaded:
    sizes, monotone offsets, sub-stage images inside their buffer."""
    try:
        tk, tn = int(meta["tk"]), int(meta["tn"])
        n_bands = -(-tn // BAND_TILES)
        n_sub = 2 * n_bands * ((tk + 1) // 2)
        rb = int(meta["record_bytes"])
        a = {k: np.asarray(arrs[k]) for k in _STREAM_ARRAYS}
    except (KeyError, TypeError, ValueError):
        raise ValueError("saved device stream: metadata or arrays missing") from None
    want = {"tiles": (np.uint8, tk * tn * 16), "row_off": (np.int32, n_bands * (tk + 1)),
            "records": (np.uint8, max(rb, 16)), "stage_counts": (np.int32, n_sub),
            "stage_offsets": (np.int32, n_sub + 1), "stage_ranges": (np.int32, 4 * n_sub)}
    for k, (dt, n) in want.items():
        if a[k].dtype != dt or a[k].size != n:
            raise ValueError(f"saved device stream: {k} has {a[k].size} x {a[k].dtype}, expected {n} x {np.dtype(dt)}")
    if a["stage_images"].dtype != np.uint8:
        raise ValueError("saved device stream: stage_images must be bytes")
    ro = a["row_off"].reshape(n_bands, tk + 1).astype(np.int64)
    if (np.diff(ro, axis=1) < 0).any() or ro.min(initial=0) < 0 or ro.max(initial=0) > rb:
        raise ValueError("saved device stream: row offsets not monotone or beyond the records")
    offs = a["stage_offsets"].view(np.uint32).astype(np.int64)
    sizes = a["stage_ranges"].view(np.uint32).astype(np.int64).reshape(n_sub, 4)[:, 0]
    if (offs % 16).any() or (np.diff(offs) < sizes).any() or offs[-1] > a["stage_images"].size:
        raise ValueError("saved device stream: sub-stage images overlap or lie outside their buffer")
    if sizes.max(initial=0) > int(meta["max_stage_bytes"]):
        raise ValueError("saved device stream: a sub-stage image exceeds the recorded maximum")


class DeviceStream:
    """GPU tile stream of one MTCMatrix on one device (built by the GPU repack)."""

    def __init__(self, mat, device):
        if not torch.cuda.is_available():
            raise RuntimeError("the MTC GEMM path needs a CUDA device (B200, sm_100a); none is available")
        lib = _lib.load()
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise ValueError(f"DeviceStream needs a CUDA device, got {self.device}")
        K, N = mat.shape
        self.K, self.N = int(K), int(N)
        ls = mat.leaf_set
        leaves, begin, tk, tn = layout.device_leaf_list(ls, self.K, self.N)
        self.tk, self.tn = tk, tn
        self.n_bands = -(-tn // BAND_TILES)
        self.exp2 = layout.choose_exp2(ls)
        self.scale_words = 1 if layout.bf16_exact(ls.scale) else 2
        dev = self.device
        arena = np.ascontiguousarray(mat.arena.raw_buffer[:max(mat.total_bytes_allocated, 1)])
        with torch.cuda.device(dev):
            d_arena = torch.from_numpy(arena).to(dev)
            d_leaves = torch.from_numpy(leaves.view(np.uint8).copy()).to(dev)
            d_begin = torch.from_numpy(begin.view(np.int32).copy()).to(dev)
            T = tk * tn
            self.tiles = torch.empty(T * 16, dtype=torch.uint8, device=dev)
            self.row_off = torch.empty(self.n_bands * (tk + 1), dtype=torch.int32, device=dev)
            scratch = torch.empty(T + 8, dtype=torch.int32, device=dev)
            out = (ctypes.c_uint64 * 2)()
            st = _stream(dev)
            _lib.check(lib.mtc_repack_plan(d_leaves.data_ptr(), d_begin.data_ptr(), tk, tn, BAND_TILES,
                                           self.scale_words, self.tiles.data_ptr(), self.row_off.data_ptr(),
                                           scratch.data_ptr(), out, st), "repack plan")
            self.record_bytes = int(out[0])
            self.max_row_bytes = int(out[1])
            self.records = torch.empty(max(self.record_bytes, 16), dtype=torch.uint8, device=dev)
            self.desc = _lib.StreamDesc(
                records=self.records.data_ptr(), tiles=self.tiles.data_ptr(), row_off=self.row_off.data_ptr(),
                K=self.K, N=self.N, tk=tk, tn=tn, band_tiles=BAND_TILES, exp2=self.exp2,
                record_bytes=self.record_bytes, max_row_bytes=self.max_row_bytes, scale_words=self.scale_words)
            _lib.check(lib.mtc_repack_fill(d_arena.data_ptr(), arena.nbytes, d_leaves.data_ptr(),
                                           d_begin.data_ptr(), ctypes.byref(self.desc), self.records.data_ptr(),
                                           scratch.data_ptr(), st), "repack fill")
            # sub-stage images for the tensor-core kernels (half a band, two k-tile
            # rows each): descriptors, class-sorted work list, a copy of the records
            n_sub = 2 * self.n_bands * ((tk + 1) // 2)
            self.stage_counts = torch.empty(n_sub, dtype=torch.int32, device=dev)
            self.stage_offsets = torch.empty(n_sub + 1, dtype=torch.int32, device=dev)
            self.stage_ranges = torch.empty(4 * n_sub, dtype=torch.int32, device=dev)
            st_scratch = torch.empty(n_sub + 8, dtype=torch.int32, device=dev)
            _lib.check(lib.mtc_repack_stage_plan(ctypes.byref(self.desc), self.stage_counts.data_ptr(),
                                                 self.stage_offsets.data_ptr(), self.stage_ranges.data_ptr(),
                                                 st_scratch.data_ptr(), out, st),
                       "repack stage plan")
            self.stage_images = torch.zeros(max(int(out[0]), 16), dtype=torch.uint8, device=dev)
            self.max_stage_bytes = int(out[1])
            _lib.check(lib.mtc_repack_stage_fill(ctypes.byref(self.desc), self.stage_offsets.data_ptr(),
                                                 self.stage_images.data_ptr(), st), "repack stage fill")
            self._finish(mat, len(ls))

    def _finish(self, mat, n_leaves: int):
        """Descriptor fields of the sub-stage images, permutations and the
        per-stream counters (shared by the repack and the upload paths)."""
        dev = self.device
        with torch.cuda.device(dev):
            self.desc.stage_images = self.stage_images.data_ptr()
            self.desc.stage_counts = self.stage_counts.data_ptr()
            self.desc.stage_offsets = self.stage_offsets.data_ptr()
            self.desc.stage_ranges = self.stage_ranges.data_ptr()
            self.desc.max_stage_bytes = self.max_stage_bytes
            self.row_perm = None if mat.row_perm is None else torch.from_numpy(
                np.asarray(mat.row_perm, dtype=np.int32)).to(dev)
            self.col_perm = None if mat.col_perm is None else torch.from_numpy(
                np.asarray(mat.col_perm, dtype=np.int32)).to(dev)
            self.col_perm_inv = None
            if mat.col_perm is not None:
                inv = np.empty(self.N, dtype=np.int32)
                inv[np.asarray(mat.col_perm)] = np.arange(self.N, dtype=np.int32)
                self.col_perm_inv = torch.from_numpy(inv).to(dev)
            self.counters = torch.zeros(self.n_bands, dtype=torch.int32, device=dev)
            self.decode_counters = torch.zeros(2 * self.n_bands, dtype=torch.int32, device=dev)
            self.status = torch.zeros(1, dtype=torch.int32, device=dev)
        self._ws = {}
        self.n_leaves = n_leaves
        self.source = getattr(self, "source", "repack")  # "repack" or "file" (uploaded by from_buffers)
        self._mat = mat          # host layout, for the strip stream built on first use
        self._strip = None
        # decode kernel for M <= 4: "strip" (mma.sync over the strip stream,
        # built on first use) or "tensor" (tcgen05 over the sub-stage images)
        self.decode_kernel = "strip"

    def with_perms(self, row_perm, col_perm) -> "DeviceStream":
        """The same packed stream (buffers shared, nothing repacked) with other
        row / column permutations (numpy int arrays or None), e.g. after
        folding a permutation into a neighbouring layer."""
        import copy

        new = copy.copy(self)
        new.desc = _lib.StreamDesc.from_buffer_copy(self.desc)
        dev = self.device
        with torch.cuda.device(dev):
            new.row_perm = None if row_perm is None else torch.from_numpy(
                np.asarray(row_perm, dtype=np.int32)).to(dev)
            new.col_perm = None if col_perm is None else torch.from_numpy(
                np.asarray(col_perm, dtype=np.int32)).to(dev)
            new.col_perm_inv = None
            if col_perm is not None:
                inv = np.empty(self.N, dtype=np.int32)
                inv[np.asarray(col_perm)] = np.arange(self.N, dtype=np.int32)
                new.col_perm_inv = torch.from_numpy(inv).to(dev)
            new.counters = torch.zeros_like(self.counters)
            new.decode_counters = torch.zeros_like(self.decode_counters)
            new.status = torch.zeros_like(self.status)
        new._ws = {}
        new._strip = self._strip  # read-only on the device: shared
        return new

    # ------------------------------------------------------------------ saving / loading
    def export_buffers(self):
        """(metadata, name -> numpy array) of the device stream, for the
        on-disk format (tensorpack_b200.core.fileformat)."""
        meta = {"version": STREAM_FORMAT_VERSION, "band_tiles": BAND_TILES, "K": self.K, "N": self.N,
                "tk": self.tk, "tn": self.tn, "exp2": self.exp2, "scale_words": self.scale_words,
                "record_bytes": self.record_bytes, "max_row_bytes": self.max_row_bytes,
                "max_stage_bytes": self.max_stage_bytes}
        arrs = {name: getattr(self, name).cpu().numpy() for name in _STREAM_ARRAYS}
        return meta, arrs

    @classmethod
    def from_buffers(cls, mat, device, meta: dict, arrs: dict) -> "DeviceStream":
        """Upload a saved stream (checked by ``stream_compatible`` and
        ``check_stream_buffers``) instead of repacking."""
        if not torch.cuda.is_available():
            raise RuntimeError("the MTC GEMM path needs a CUDA device (B200, sm_100a); none is available")
        _lib.load()
        check_stream_buffers(meta, arrs)
        self = cls.__new__(cls)
        self.source = "file"
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise ValueError(f"DeviceStream needs a CUDA device, got {self.device}")
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        self.K, self.N = int(meta["K"]), int(meta["N"])
        self.tk, self.tn = int(meta["tk"]), int(meta["tn"])
        self.n_bands = -(-self.tn // BAND_TILES)
        self.exp2, self.scale_words = int(meta["exp2"]), int(meta["scale_words"])
        self.record_bytes, self.max_row_bytes = int(meta["record_bytes"]), int(meta["max_row_bytes"])
        self.max_stage_bytes = int(meta["max_stage_bytes"])
        with torch.cuda.device(self.device):
            for name in _STREAM_ARRAYS:
                a = np.ascontiguousarray(arrs[name])
                setattr(self, name, torch.from_numpy(a.copy()).to(self.device))
        self.desc = _lib.StreamDesc(
            records=self.records.data_ptr(), tiles=self.tiles.data_ptr(), row_off=self.row_off.data_ptr(),
            K=self.K, N=self.N, tk=self.tk, tn=self.tn, band_tiles=BAND_TILES, exp2=self.exp2,
            record_bytes=self.record_bytes, max_row_bytes=self.max_row_bytes, scale_words=self.scale_words)
        self._finish(mat, mat.num_leaves)
        return self

    # ------------------------------------------------------------------
    @property
    def device_bytes(self) -> int:
        """Bytes of the device format (records + descriptors + row offsets)."""
        return self.record_bytes + self.tiles.numel() + 4 * self.row_off.numel()

    def dequant(self, original_order: bool = True, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Exact fp32 reconstruction (bit-identical to the reference dequant)."""
        lib = _lib.load()
        if out is None:
            out = torch.empty(self.K, self.N, dtype=torch.float32, device=self.device)
        assert out.shape == (self.K, self.N) and out.dtype == torch.float32 and out.stride(1) == 1
        pr = self.row_perm if original_order else None
        pc = self.col_perm if original_order else None
        _lib.check(lib.mtc_dequant(ctypes.byref(self.desc), _ptr(pr), _ptr(pc), out.data_ptr(), out.stride(0),
                                   _stream(self.device)), "dequant")
        return out

    def _workspace(self, M: int, rows_per_unit: int) -> torch.Tensor:
        lib = _lib.load()
        need = int(lib.mtc_gemv_workspace_bytes(ctypes.byref(self.desc), M, rows_per_unit))
        key = (M > 8, rows_per_unit)
        ws = self._ws.get(key)
        if ws is None or ws.numel() * 4 < need:
            ws = torch.empty(max(need // 4, 1), dtype=torch.float32, device=self.device)
            self._ws[key] = ws
        return ws

    def gemv(self, X: torch.Tensor, Y: torch.Tensor, rows_per_unit: int = 0) -> torch.Tensor:
        """Y[:M] = X @ W for M <= 16 (split-K streaming kernel)."""
        lib = _lib.load()
        M = X.shape[0]
        ws = self._workspace(M, rows_per_unit)
        _lib.check(lib.mtc_gemv(ctypes.byref(self.desc), X.data_ptr(), M, X.stride(0), _ptr(self.row_perm),
                                _ptr(self.col_perm), Y.data_ptr(), Y.stride(0), rows_per_unit, ws.data_ptr(),
                                ws.numel() * 4, self.counters.data_ptr(), self.status.data_ptr(),
                                _stream(self.device)), "gemv")
        return Y

    def decode(self, X: torch.Tensor, Y: torch.Tensor, ep: Optional[_lib.Epilogue] = None) -> torch.Tensor:
        """Y[:M] = X @ W for M <= 16 (tensor-core decode kernel); ``ep`` from
        ``epilogue()`` fuses a bias and activation into the output."""
        lib = _lib.load()
        M = X.shape[0]
        need = int(lib.mtc_decode_workspace_bytes(ctypes.byref(self.desc), M))
        ws = self._ws.get("decode")
        if ws is None or ws.numel() < need:
            ws = torch.empty(max(need, 256), dtype=torch.uint8, device=self.device)
            self._ws["decode"] = ws
        _lib.check(lib.mtc_decode(ctypes.byref(self.desc), X.data_ptr(), M, X.stride(0), _ptr(self.row_perm),
                                  _ptr(self.col_perm), Y.data_ptr(), Y.stride(0), ws.data_ptr(), ws.numel(),
                                  self.decode_counters.data_ptr(), self.status.data_ptr(), _ep(ep),
                                  _stream(self.device)), "decode")
        return Y

    def strip(self, wide: bool = False, batch_bytes: Optional[int] = None,
              batch_steps: Optional[int] = None, merge_modes: bool = False) -> "DeviceStrip":
        """The strip stream of this matrix on this device (the decode layout
        for M <= 4), built on the host and uploaded at first use.  ``wide``
        gives the MTC_STRIP_WIDE form, ``merge_modes`` packs P2 / P6 items
        with the P3 / P8 decoders; ``batch_bytes`` / ``batch_steps``
        override the batch record limits.  The decode uses the default
        stream; the other forms are built on request (for measurements)."""
        from ..core import strip as _strip

        if wide or merge_modes or batch_bytes is not None or batch_steps is not None:
            key = (wide, merge_modes, batch_bytes or _strip.BATCH_BYTES, batch_steps or _strip.BATCH_STEPS)
            other = self.__dict__.setdefault("_strip_other", {})
            if key not in other:
                other[key] = DeviceStrip(_strip.build_host(self._mat, key[2], key[3], wide=wide,
                                                           merge_modes=merge_modes), self.device)
            return other[key]
        if self._strip is None:
            self._strip = DeviceStrip(self._mat.host_strip(), self.device)
        return self._strip

    def strip_fits(self, M: int) -> bool:
        """Whether the strip kernel can run this matrix at M tokens (its
        gathered activations and batch slots fit shared memory; K up to
        about 24K at M = 3..4, about 100K at M = 1)."""
        fits = self.__dict__.setdefault("_strip_fits", {})
        if M not in fits:
            fits[M] = bool(_lib.load().mtc_strip_fits(ctypes.byref(self.strip().desc_for(M)), M))
        return fits[M]

    def decode_strip(self, X: torch.Tensor, Y: torch.Tensor, ep: Optional[_lib.Epilogue] = None) -> torch.Tensor:
        """Y[:M] = X @ W for M <= 4 (mma.sync kernel over the strip stream);
        ``ep`` from ``epilogue()`` fuses a bias and activation."""
        lib = _lib.load()
        st = self.strip()
        _lib.check(lib.mtc_strip_decode(ctypes.byref(st.desc_for(X.shape[0])), X.data_ptr(), X.shape[0], X.stride(0),
                                        _ptr(self.row_perm), _ptr(self.col_perm), Y.data_ptr(), Y.stride(0),
                                        self.status.data_ptr(), _ep(ep), _stream(self.device)), "strip decode")
        return Y

    def prefill_workspace(self, M: int) -> torch.Tensor:
        lib = _lib.load()
        permuted = 1 if self.col_perm_inv is not None else 0
        need = int(lib.mtc_prefill_workspace_bytes(ctypes.byref(self.desc), M, permuted))
        ws = self._ws.get("prefill")
        if ws is None or ws.numel() < need:
            ws = torch.empty(max(need, 256), dtype=torch.uint8, device=self.device)
            self._ws["prefill"] = ws
        return ws

    def prefill(self, X: torch.Tensor, Y: torch.Tensor, ep: Optional[_lib.Epilogue] = None) -> torch.Tensor:
        """Y = X @ W for any M (fused dequant + tcgen05 kernel; used for M > 16)."""
        lib = _lib.load()
        M = X.shape[0]
        ws = self.prefill_workspace(M)
        _lib.check(lib.mtc_gemm_prefill(ctypes.byref(self.desc), X.data_ptr(), M, X.stride(0), _ptr(self.row_perm),
                                        _ptr(self.col_perm_inv), Y.data_ptr(), Y.stride(0), ws.data_ptr(),
                                        ws.numel(), self.status.data_ptr(), _ep(ep), _stream(self.device)),
                   "prefill")
        return Y

    # The three prefill stages, for callers that time or fuse them separately.
    def prefill_gather(self, X: torch.Tensor):
        lib = _lib.load()
        ws = self.prefill_workspace(X.shape[0])
        _lib.check(lib.mtc_prefill_gather(ctypes.byref(self.desc), X.data_ptr(), X.shape[0], X.stride(0),
                                          _ptr(self.row_perm), ws.data_ptr(), ws.numel(), self.status.data_ptr(),
                                          _stream(self.device)), "prefill gather")

    def prefill_gemm(self, M: int, Y: torch.Tensor, ep: Optional[_lib.Epilogue] = None):
        lib = _lib.load()
        ws = self.prefill_workspace(M)
        permuted = 1 if self.col_perm_inv is not None else 0
        _lib.check(lib.mtc_prefill_gemm(ctypes.byref(self.desc), M, Y.data_ptr(), Y.stride(0), permuted,
                                        ws.data_ptr(), ws.numel(), self.status.data_ptr(),
                                        None if permuted else _ep(ep), _stream(self.device)), "prefill gemm")

    def prefill_scatter(self, M: int, Y: torch.Tensor, ep: Optional[_lib.Epilogue] = None):
        if self.col_perm_inv is None:
            return
        lib = _lib.load()
        ws = self.prefill_workspace(M)
        _lib.check(lib.mtc_prefill_scatter(ctypes.byref(self.desc), M, self.col_perm_inv.data_ptr(), Y.data_ptr(),
                                           Y.stride(0), ws.data_ptr(), ws.numel(), _ep(ep), _stream(self.device)),
                   "prefill scatter")

    def matmul(self, X: torch.Tensor, Y: torch.Tensor, ep: Optional[_lib.Epilogue] = None) -> torch.Tensor:
        """Y = X @ W (+ the fused epilogue ``ep``): the strip-stream decode for
        M <= 4 when it fits (``decode_kernel = "tensor"`` selects the tcgen05
        decode), the tcgen05 decode for M <= 16, the tensor-core prefill
        kernel above."""
        M = X.shape[0]
        if M <= STRIP_MAX_M and self.decode_kernel == "strip" and self.strip_fits(M):
            return self.decode_strip(X, Y, ep)
        if M <= DECODE_MAX_M:
            return self.decode(X, Y, ep)
        return self.prefill(X, Y, ep)

    def check_status(self):
        """Raise if a kernel reported a runtime problem (synchronises).

        A call that gave up part-way can leave split-K tickets counted, so
        both ticket arrays are cleared with the status word: the next call
        starts from the zero state the kernels expect."""
        v = int(self.status.item())
        if v:
            self.status.zero_()
            self.counters.zero_()
            self.decode_counters.zero_()
            bits = []
            if v & _lib.STATUS_TIMEOUT:
                bits.append("pipeline wait timed out")
            if v & _lib.STATUS_X_RANGE:
                bits.append("|X| exceeds the fp16 range (65504) of the tensor-core path")
            if v & _lib.STATUS_BAD_STREAM:
                bits.append("tile stream failed a bounds check")
            raise RuntimeError("MTC kernel status: " + "; ".join(bits))


class DeviceStrip:
    """The strip stream of one matrix on one device: batch records, batch
    offsets and per-strip batch ranges (uploaded from a HostStripStream),
    the kernel's static schedules for this device's SM count (one with more
    warps for M = 1, one for M = 2..4), and their C descriptors."""

    def __init__(self, hs, device, n_warps: Optional[int] = None):
        from ..core import strip as _strip

        dev = torch.device(device)
        if dev.index is None:
            dev = torch.device("cuda", torch.cuda.current_device())
        sms = max(int(_lib.load().mtc_device_sm_count(dev.index)), 1)
        warps = (n_warps, n_warps) if n_warps else (_strip.WARPS_M1, _strip.WARPS)
        with torch.cuda.device(dev):
            self.stream = torch.from_numpy(hs.stream).to(dev)
            self.batch_off = torch.from_numpy(hs.batch_off.view(np.int32)).to(dev)
            self.strip_batch = torch.from_numpy(hs.strip_batch.view(np.int32)).to(dev)
        self.host = hs
        self.device = dev
        self._descs, self._keep = [], []
        for nw in dict.fromkeys(warps):  # distinct warp counts, in order
            sched = hs.schedule(sms, nw)
            with torch.cuda.device(dev):
                arrays = [torch.from_numpy(a.view(np.int32)).to(dev) for a in
                          (sched.work, sched.warp_work, sched.red, sched.cta_red)]
            self._keep.append((sched, arrays))
            self._descs.append(hs.desc(self.stream.data_ptr(), self.batch_off.data_ptr(), self.strip_batch.data_ptr(),
                                       sched, [a.data_ptr() for a in arrays]))
        self.sched = self._keep[-1][0]
        self.desc = self._descs[-1]      # M = 2..4 (and any M)
        self.desc_m1 = self._descs[0]    # M = 1

    def desc_for(self, M: int) -> _lib.StripDesc:
        """The descriptor whose schedule serves M tokens."""
        return self.desc_m1 if M == 1 else self.desc

    @property
    def stream_bytes(self) -> int:
        return int(self.host.batch_off[-1])
