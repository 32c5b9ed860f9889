"""Drop-in ``MTCMatrix`` / ``mtc_gemm`` backed by sm_100a CUDA kernels.

Mirrors ``mtc.kernels.gemm`` of the reference (mtc/kernels/gemm.py:217-574):
the same class and function names, constructor arguments, properties and
exceptions.  Differences, all additive:

* an ``MTCMatrix`` can also hold a quadtree allocation (MTC-QT leaves of edge
  32..4, optionally with the MTC-QT-P row/column permutation):
  ``MTCMatrix.from_qt_allocation(W, alloc)``;
* ``mtc_gemm(X, W)`` accepts activations X (numpy or a CUDA torch tensor) as
  the left operand, besides the reference's ``mtc_gemm(A, B)`` with two
  packed matrices;
* the multiply, the dequantisation (``to_array``) and the repack into the
  device tile stream run on the GPU.  There is no CPU fallback: without CUDA
  these raise.
"""

from __future__ import annotations

from typing import Optional, Sequence, Tuple

import numpy as np

from ..core import layout
from ..core.arena import MemoryArena
from ..core.types import META_BITS, PrecisionMode

_LEGACY_QMAX = {PrecisionMode.P2: 1.0, PrecisionMode.P4: 7.0, PrecisionMode.P8: 127.0, PrecisionMode.P16: 32767.0}
_LEGACY_CLIP = {PrecisionMode.P2: (-2, 1), PrecisionMode.P4: (-8, 7), PrecisionMode.P8: (-128, 127),
                PrecisionMode.P16: (-32768, 32767)}


def _legacy_select(block: np.ndarray, epsilon: float):
    """Lowest of P2/P4/P8 whose block reconstruction error is <= epsilon, else
    (P16, 1.0) (mtc/core/precision.py:11-74)."""
    arr = np.asarray(block, dtype=np.float32)
    max_abs = float(np.max(np.abs(arr)))
    norm = float(np.linalg.norm(arr))
    for p in (PrecisionMode.P2, PrecisionMode.P4, PrecisionMode.P8):
        if max_abs < 1e-8:
            return p, 1.0
        sc = max_abs / _LEGACY_QMAX[p]
        lo, hi = _LEGACY_CLIP[p]
        rec = np.clip(np.round(arr / sc), lo, hi).astype(np.int8).astype(np.float32) * sc
        err = 0.0 if norm < 1e-8 else float(np.linalg.norm(arr.astype(np.float32) - rec.astype(np.float32))) / norm
        if err <= epsilon:
            return p, sc
    return PrecisionMode.P16, 1.0


class MTCMatrix:
    """An (H, W) matrix of MTC blocks whose payloads live in a byte arena.

    Reference layout (gemm.py:217-238): ``offsets``, ``precisions`` and
    ``scales`` are (H/Bs, W/Bs) grids for a fixed ``block_size``.  For a
    quadtree matrix they are per-leaf vectors in canonical order (32x32 tiles
    row-major, Z order inside a tile) and ``leaf_rows`` / ``leaf_cols`` /
    ``leaf_sizes`` give each leaf's placement in the stored (permuted) matrix.
    """

    def __init__(
        self,
        shape: Tuple[int, int],
        block_size: int,
        arena: MemoryArena,
        offsets: np.ndarray,
        precisions: np.ndarray,
        scales: np.ndarray,
        pointer_tensor=None,
        *,
        leaf_rows: Optional[np.ndarray] = None,
        leaf_cols: Optional[np.ndarray] = None,
        leaf_sizes: Optional[np.ndarray] = None,
        sizes: Optional[Sequence[int]] = None,
        row_perm: Optional[np.ndarray] = None,
        col_perm: Optional[np.ndarray] = None,
    ):
        self.shape = tuple(int(x) for x in shape)
        self.block_size = int(block_size)
        self.arena = arena
        self.offsets = offsets
        self.precisions = precisions
        self.scales = scales
        self.pointer_tensor = pointer_tensor
        self.leaf_rows = leaf_rows
        self.leaf_cols = leaf_cols
        self.leaf_sizes = leaf_sizes
        self.sizes = tuple(sizes) if sizes is not None else (self.block_size,)
        self.row_perm = None if row_perm is None else np.asarray(row_perm, dtype=np.int64)
        self.col_perm = None if col_perm is None else np.asarray(col_perm, dtype=np.int64)
        self._device = {}

    # ------------------------------------------------------------------ reference properties
    @property
    def num_blocks(self) -> Tuple[int, ...]:
        return self.offsets.shape

    @property
    def total_bytes_allocated(self) -> int:
        return self.arena.bytes_allocated

    @property
    def average_bits_per_element(self) -> float:
        n = self.shape[0] * self.shape[1]
        return 0.0 if n == 0 else (self.total_bytes_allocated * 8.0) / n

    # ------------------------------------------------------------------ new properties
    @property
    def is_quadtree(self) -> bool:
        return self.leaf_rows is not None

    @property
    def leaf_set(self) -> layout.LeafSet:
        if self.is_quadtree:
            return layout.LeafSet(np.asarray(self.leaf_rows, np.int64), np.asarray(self.leaf_cols, np.int64),
                                  np.asarray(self.leaf_sizes, np.int64), np.asarray(self.precisions, np.uint8),
                                  np.asarray(self.scales, np.float32), np.asarray(self.offsets, np.int64))
        return layout.leaves_from_grid(np.asarray(self.precisions), np.asarray(self.scales), self.block_size,
                                       np.asarray(self.offsets))

    @property
    def num_leaves(self) -> int:
        return int(np.asarray(self.precisions).size)

    @property
    def scale_format(self) -> str:
        return "bf16" if layout.bf16_exact(np.asarray(self.scales)) else "fp32"

    @property
    def accounted_bits(self) -> int:
        """Bits of the stored format as the allocators count them: payload +
        scale/mode per leaf + split flags + permutation indices
        (quadtree.py:97-117, permutation.py:49-51, allocation.py:197)."""
        ls = self.leaf_set
        bits = int((ls.mode.astype(np.int64) * ls.size ** 2).sum())
        bits += META_BITS[self.scale_format] * len(ls)
        if self.is_quadtree:
            bits += layout.flag_bits(ls, self.sizes)
        K, N = self.shape
        bits += layout.index_bits(K, N, self.row_perm is not None, self.col_perm is not None)
        return bits

    # ------------------------------------------------------------------ constructors
    @classmethod
    def from_numpy(cls, matrix: np.ndarray, block_size: int = 16, precision_mode: Optional[PrecisionMode] = None,
                   epsilon: float = 0.05, arena: Optional[MemoryArena] = None,
                   use_pointer_hierarchy: bool = True) -> "MTCMatrix":
        """Legacy per-block adaptive packing (gemm.py:255-328, microtensor.py:64-176).

        The pointer-tensor DAG of the reference is not built (``pointer_tensor``
        stays None); payload bytes, offsets and scales match the reference."""
        arr = np.asarray(matrix, dtype=np.float32)
        H, W = arr.shape
        Bs = block_size
        assert H % Bs == 0 and W % Bs == 0, f"Dimensions ({H}, {W}) must be divisible by block_size {Bs}"
        if arena is None:
            arena = MemoryArena(capacity_bytes=max(1024 * 1024, H * W * 2))
        nbh, nbw = H // Bs, W // Bs
        offsets = np.zeros((nbh, nbw), dtype=np.uint32)
        precisions = np.zeros((nbh, nbw), dtype=np.uint8)
        scales = np.zeros((nbh, nbw), dtype=np.float32)
        for bi in range(nbh):
            for bj in range(nbw):
                block = arr[bi * Bs:(bi + 1) * Bs, bj * Bs:(bj + 1) * Bs]
                if precision_mode is not None:
                    p = PrecisionMode(precision_mode)
                    max_abs = float(np.max(np.abs(block)))
                    sc = (max_abs / _LEGACY_QMAX[p] if max_abs > 1e-7 else 1.0) if p in _LEGACY_QMAX else 1.0
                else:
                    p, sc = _legacy_select(block, epsilon)
                if p not in _LEGACY_CLIP:
                    raise ValueError(f"Unsupported precision: {p}")
                inv = 1.0 / sc if sc != 0.0 else 1.0
                lo, hi = _LEGACY_CLIP[p]
                q = np.clip(np.round(block * inv), lo, hi).astype(np.int64).reshape(1, -1)
                packed = layout.pack_bitstream(q, int(p))[0]
                offsets[bi, bj] = arena.write_bytes(packed, alignment=2 if p == PrecisionMode.P16 else 1)
                precisions[bi, bj] = int(p)
                scales[bi, bj] = sc
        return cls((H, W), Bs, arena, offsets, precisions, scales, None)

    @classmethod
    def from_allocation(cls, matrix: np.ndarray, modes: np.ndarray, scales: np.ndarray,
                        block_size: int) -> "MTCMatrix":
        """Pack a matrix given per-block modes and scales (gemm.py:432-488):
        row-major block order, P0 blocks occupy zero bytes."""
        arr = np.asarray(matrix, dtype=np.float32)
        H, W = arr.shape
        Bs = block_size
        nbh, nbw = H // Bs, W // Bs
        modes = np.asarray(modes, dtype=np.uint8).reshape(nbh, nbw)
        scales = np.asarray(scales, dtype=np.float32).reshape(nbh, nbw)
        ls = layout.leaves_from_grid(modes, scales, Bs)
        buf, offs = layout.pack_leaves(arr, ls)
        total = int(ls.payload_bytes.sum())
        arena = MemoryArena(capacity_bytes=max(total, 1))
        base = arena.allocate(total, alignment=2)
        arena.raw_buffer[base:base + total] = buf[:total]
        offsets = (offs + base).astype(np.uint32).reshape(nbh, nbw)
        return cls((H, W), Bs, arena, offsets, modes.copy(),
                   np.where(modes == 0, 0.0, scales).astype(np.float32), None)

    @classmethod
    def from_qt_allocation(cls, W: np.ndarray, alloc, codes: Optional[np.ndarray] = None) -> "MTCMatrix":
        """Pack an MTC-QT (QTAllocation) or MTC-QT-P (PermutedQTAllocation)
        allocation of W (original channel order).

        Leaves are stored in canonical order (32x32 tiles row-major, Z order
        inside a tile) with the reference's per-mode payload packing; the
        permutation, if any, is kept for the GEMM's gather / scatter.
        ``codes`` (stored order, same shape as W) packs explicit integer codes
        instead of rint(W / s), e.g. from GPTQ."""
        W = np.asarray(W, dtype=np.float32)
        inner = getattr(alloc, "inner", None)
        if inner is not None:
            pr, pc = np.asarray(alloc.row_perm), np.asarray(alloc.col_perm)
            Wp = W[pr][:, pc]
        else:
            inner, pr, pc, Wp = alloc, None, None, W
        sizes = tuple(int(s) for s in inner.sizes)
        for s in sizes:
            if s not in layout.SUPPORTED_LEAF_SIZES:
                raise ValueError(f"quadtree level {s} not supported (levels must be within 32..4)")
        ls = layout.leaves_from_quadtree(sizes, inner.leaf, inner.modes, inner.scales)
        ls.scale = np.where(ls.mode == 0, np.float32(0), ls.scale).astype(np.float32)
        buf, offs = layout.pack_leaves(Wp, ls, codes)
        total = int(ls.payload_bytes.sum())
        arena = MemoryArena(capacity_bytes=max(total, 1))
        base = arena.allocate(total, alignment=2)
        arena.raw_buffer[base:base + total] = buf[:total]
        return cls(W.shape, sizes[0], arena, (offs + base).astype(np.uint32), ls.mode.copy(), ls.scale.copy(), None,
                   leaf_rows=ls.row, leaf_cols=ls.col, leaf_sizes=ls.size, sizes=sizes, row_perm=pr, col_perm=pc)

    # ------------------------------------------------------------------ device side
    def device_stream(self, device=None):
        """The GPU tile stream of this matrix on ``device`` (repacked once)."""
        import torch

        from .device import DeviceStream

        dev = torch.device(device if device is not None else "cuda")
        if dev.type == "cuda" and dev.index is None:
            dev = torch.device("cuda", torch.cuda.current_device())
        key = str(dev)
        ds = self._device.get(key)
        if ds is None:
            ds = DeviceStream(self, dev)
            self._device[key] = ds
        return ds

    def attach_device_stream(self, ds) -> None:
        """Use an already built device stream (e.g. uploaded from a file)."""
        self._device[str(ds.device)] = ds

    def host_strip(self):
        """The default strip stream of this matrix (the decode layout for
        M <= 4) in host memory: built on first use, or the one loaded from a
        file (tensorpack_b200.core.strip)."""
        hs = getattr(self, "_host_strip", None)
        if hs is None:
            from ..core import strip as _strip

            hs = _strip.build_host(self)
            self._host_strip = hs
        return hs

    def attach_host_strip(self, hs) -> None:
        """Use an already built default strip stream (e.g. read from a file)."""
        from ..core import strip as _strip

        if hs.flags != 0 or hs.max_batch_bytes > _strip.BATCH_BYTES:
            raise ValueError("attach_host_strip: only the default strip form can be attached")
        self._host_strip = hs

    # ------------------------------------------------------------------ files
    def save(self, path, *, include_stream: bool = False, device=None, include_strip: bool = False) -> None:
        """Write this matrix to a versioned ``.mtcpk`` file
        (tensorpack_b200.core.fileformat); ``include_stream`` also stores the
        device tile stream so that loading skips the repack, and
        ``include_strip`` the decode kernel's strip stream (built on the
        host, no GPU needed)."""
        from ..core.fileformat import save_mtc

        save_mtc(path, self, include_stream=include_stream, device=device, include_strip=include_strip)

    @classmethod
    def load(cls, path, *, device=None, use_stream: bool = True, mmap: bool = False) -> "MTCMatrix":
        """Read a matrix written by ``save`` (raises ValueError on a corrupt,
        truncated or foreign file)."""
        from ..core.fileformat import load_mtc

        mat = load_mtc(path, device=device, use_stream=use_stream, mmap=mmap)
        if not isinstance(mat, cls):
            raise ValueError(f"{path} holds a bundle of {len(mat)} matrices; use fileformat.load_mtc")
        return mat

    def to_tensor(self, device=None):
        """Exact fp32 dequantisation on the GPU, original channel order."""
        return self.device_stream(device).dequant(original_order=True)

    def to_array(self) -> np.ndarray:
        """Reconstruct the full float32 matrix (gemm.py:510-538), bit-exact, on the GPU."""
        return self.to_tensor().cpu().numpy()


def _as_cuda_f32(X, device):
    import torch

    if isinstance(X, np.ndarray):
        return torch.from_numpy(np.ascontiguousarray(X, dtype=np.float32)).to(device), True
    if not isinstance(X, torch.Tensor):
        raise TypeError(f"mtc_gemm: unsupported operand type {type(X).__name__}")
    if X.device.type != "cuda":
        raise ValueError("mtc_gemm: activations must be a CUDA tensor (no CPU path)")
    X = X.float() if X.dtype != torch.float32 else X
    if X.dim() != 2 or X.stride(1) != 1:
        X = X.contiguous()
    return X, False


def gemm_into(X, W: MTCMatrix, Y):
    """Y = X @ W on the GPU (X, Y CUDA fp32, row-major)."""
    return W.device_stream(X.device).matmul(X, Y)


def gemm_fused(X, W: MTCMatrix, bias=None, activation: Optional[str] = None, Y=None):
    """Y = act(X @ W + bias) with the bias add and activation fused into the
    kernel that writes Y (the decode reduction, the prefill epilogue or the
    column scatter of a permuted matrix): one pass over the output.

    X: (M, K) CUDA tensor (fp32, or converted); bias: None or N floats (numpy
    or tensor) in the column order of Y; activation: None, "relu", "silu" or
    "gelu_tanh".  Returns Y (CUDA fp32)."""
    import torch

    from .device import epilogue

    dev = X.device if isinstance(X, torch.Tensor) else torch.device("cuda", torch.cuda.current_device())
    Xd, _ = _as_cuda_f32(X, dev)
    M, K = Xd.shape
    K2, N = W.shape
    assert K == K2, f"Shape mismatch: {tuple(Xd.shape)} vs {W.shape}"
    b = None
    if bias is not None:
        b = torch.as_tensor(bias, dtype=torch.float32, device=dev).reshape(-1).contiguous()
        if b.numel() != N:
            raise ValueError(f"bias has {b.numel()} values, the output {N} columns")
    if Y is None:
        Y = torch.empty(M, N, dtype=torch.float32, device=dev)
    if M:
        W.device_stream(dev).matmul(Xd, Y, epilogue(b, activation))
    return Y


class HostGemm:
    """Y = X @ W for activations and results in (pinned) host memory, with
    the host->device copy, the GEMM and the device->host copy of consecutive
    row chunks overlapped on three CUDA streams: the PCIe copies in both
    directions and the kernels run at the same time instead of one after the
    other.  Device buffers (two chunks) are allocated once per shape and
    reused across calls; ``__call__`` returns once Yh holds the result.

    A chunk is ``chunk_rows`` rows (a multiple of the prefill kernel's 512-row
    pair tile by default); M <= chunk_rows runs as one chunk."""

    def __init__(self, W: MTCMatrix, device=None, chunk_rows: int = 1024):
        import torch

        self.W = W
        self.device = torch.device(device if device is not None else "cuda")
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        self.chunk_rows = int(chunk_rows)
        self.ds = W.device_stream(self.device)
        with torch.cuda.device(self.device):
            self.s_in, self.s_mm, self.s_out = (torch.cuda.Stream(self.device) for _ in range(3))
        self._bufs = None

    def _buffers(self, rows: int):
        import torch

        K, N = self.W.shape
        if self._bufs is None or self._bufs[0][0].shape[0] < rows:
            self._bufs = [(torch.empty(rows, K, dtype=torch.float32, device=self.device),
                           torch.empty(rows, N, dtype=torch.float32, device=self.device)) for _ in range(2)]
        return self._bufs

    def __call__(self, Xh, Yh=None, ep=None):
        import torch

        K, N = self.W.shape
        if Xh.device.type != "cpu" or Xh.dtype != torch.float32 or Xh.dim() != 2 or Xh.shape[1] != K:
            raise ValueError(f"HostGemm: X must be a host float32 (M, {K}) tensor")
        M = Xh.shape[0]
        if Yh is None:
            Yh = torch.empty(M, N, dtype=torch.float32, pin_memory=True)
        if Yh.shape != (M, N) or Yh.device.type != "cpu" or Yh.dtype != torch.float32:
            raise ValueError(f"HostGemm: Y must be a host float32 ({M}, {N}) tensor")
        if M == 0:
            return Yh
        cr = min(self.chunk_rows, M)
        bufs = self._buffers(cr)
        cur = torch.cuda.current_stream(self.device)
        ev = {k: [torch.cuda.Event() for _ in range(2)] for k in ("in", "mm", "out")}
        started = [False, False]
        for s in (self.s_in, self.s_mm, self.s_out):
            s.wait_stream(cur)
        for i, r0 in enumerate(range(0, M, cr)):
            r1 = min(M, r0 + cr)
            b = i & 1
            Xd, Yd = bufs[b]
            with torch.cuda.stream(self.s_in):
                if started[b]:
                    self.s_in.wait_event(ev["mm"][b])        # the chunk two back has read Xd
                Xd[:r1 - r0].copy_(Xh[r0:r1], non_blocking=True)
                ev["in"][b].record(self.s_in)
            with torch.cuda.stream(self.s_mm):
                self.s_mm.wait_event(ev["in"][b])
                if started[b]:
                    self.s_mm.wait_event(ev["out"][b])       # ... and its result left Yd
                self.ds.matmul(Xd[:r1 - r0], Yd[:r1 - r0], ep)
                ev["mm"][b].record(self.s_mm)
            with torch.cuda.stream(self.s_out):
                self.s_out.wait_event(ev["mm"][b])
                Yh[r0:r1].copy_(Yd[:r1 - r0], non_blocking=True)
                ev["out"][b].record(self.s_out)
            started[b] = True
        cur.wait_stream(self.s_out)
        cur.wait_stream(self.s_mm)
        cur.synchronize()
        self.ds.check_status()
        return Yh


def mtc_gemm(A, B):
    """GEMM with a packed right operand (gemm.py:541-574).

    * ``mtc_gemm(A: MTCMatrix, B: MTCMatrix) -> np.ndarray`` (reference form,
      used by the reference's tests and benchmark runner): both operands are
      dequantised exactly on the GPU and multiplied in fp32 (no TF32), so the
      result agrees with the reference's exact-product kernel to fp32
      summation order (its tests/test_allocation.py:83 bar of 1e-5).  The
      activation form below is the fused hot path.
    * ``mtc_gemm(X, W: MTCMatrix)`` with X an (M, K) numpy array or CUDA
      tensor: returns numpy for numpy input, a CUDA fp32 tensor otherwise.
    """
    import torch

    if not isinstance(B, MTCMatrix):
        raise TypeError("mtc_gemm: the right operand must be an MTCMatrix")
    K2, N = B.shape
    if isinstance(A, MTCMatrix):
        M, K = A.shape
        assert K == K2, f"Shape mismatch: {A.shape} vs {B.shape}"
        assert A.block_size == B.block_size, "Block size mismatch"
        dev = torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available() else None
        if dev is None:
            raise RuntimeError("mtc_gemm needs a CUDA device (B200, sm_100a); none is available")
        Ad, Bd = A.to_tensor(dev), B.to_tensor(dev)
        prev = torch.backends.cuda.matmul.allow_tf32
        torch.backends.cuda.matmul.allow_tf32 = False
        try:
            Y = Ad @ Bd
        finally:
            torch.backends.cuda.matmul.allow_tf32 = prev
        return Y.cpu().numpy()
    dev = A.device if isinstance(A, torch.Tensor) else (
        torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available() else None)
    if dev is None:
        raise RuntimeError("mtc_gemm needs a CUDA device (B200, sm_100a); none is available")
    X, was_numpy = _as_cuda_f32(A, dev)
    M, K = X.shape
    assert K == K2, f"Shape mismatch: {tuple(X.shape)} vs {B.shape}"
    Y = torch.empty(M, N, dtype=torch.float32, device=X.device)
    if M:
        gemm_into(X, B, Y)
    if was_numpy:
        B.device_stream(X.device).check_status()
        return Y.cpu().numpy()
    return Y
