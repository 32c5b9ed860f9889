"""GPU MTC-QT / MTC-QT-P allocation (input producer of the packed GEMM).

The offline allocators of the reference (mtc/core/quadtree.py:72-154,
mtc/core/permutation.py:82-105) spend nearly all their time in the per-block
scale search (a Numba kernel, mtc/core/allocation.py:106-136); on a 4096 x
14336 layer that takes minutes on the host.  Here the search runs in the
``mtc_rd_search`` CUDA kernel (bit-identical distortions and scales) and the
Lagrangian tree pruning plus the bisection on lambda run as fp64 tensor ops
on the same device, so a Llama-sized layer is allocated in seconds.

The interfaces mirror the reference: ``QuadtreeRD(W, importance, sizes,
modes, scale_format).select(bits_per_element)`` returns an allocation with
``sizes / leaf / modes / scales / total_bits`` (QTAllocation fields) and
``PermutedQuadtreeRD`` adds ``row_perm / col_perm`` (PermutedQTAllocation).
The P0 distortion (a plain weighted sum of squares) is summed in a different
order than numpy's einsum, so a P0-versus-other tie can, rarely, resolve
differently from the reference; everything else follows it step for step.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass, field
from math import ceil, log2
from typing import Dict, Optional, Sequence, Tuple

import numpy as np
import torch

from .. import _lib

DEFAULT_MODES = (0, 2, 3, 4, 5, 6, 8, 16)
META_BITS = {"fp32": 40, "bf16": 24}
FLAG_BITS = 1
_ALPHA_GRID = {2: (0.20, 33), 3: (0.30, 29), 4: (0.40, 25), 5: (0.50, 21), 6: (0.60, 17), 8: (0.80, 9)}


def alpha_grid(mode: int) -> np.ndarray:
    """Clipping ratios tried per mode (mtc/core/allocation.py:67-75)."""
    if mode == 16:
        return np.array([1.0], dtype=np.float32)
    lo, n = _ALPHA_GRID[mode]
    return np.linspace(lo, 1.00, n).astype(np.float32)


@dataclass
class Allocation:
    """QTAllocation fields (mtc/core/quadtree.py:55-61); grids are numpy.
    ``dequant`` (the exact reconstruction, quadtree.py:157-171) is computed
    on first access by the GPU dequant kernel from the matrix the allocation
    was made for."""
    sizes: Tuple[int, ...]
    leaf: Dict[int, np.ndarray]
    modes: Dict[int, np.ndarray]
    scales: Dict[int, np.ndarray]
    total_bits: int
    shape: Tuple[int, int]
    source: Optional[np.ndarray] = field(default=None, repr=False)  # W the allocation was made for
    _dequant: Optional[np.ndarray] = field(default=None, repr=False)

    @property
    def bits_per_element(self) -> float:
        return self.total_bits / (self.shape[0] * self.shape[1])

    @property
    def dequant(self) -> np.ndarray:
        if self._dequant is None:
            if self.source is None:
                raise ValueError("this allocation does not hold its matrix; use qt_dequant(W, ...)")
            self._dequant = _gpu_dequant(self.source, self)
        return self._dequant

    def leaf_area_fraction(self) -> Dict[int, float]:
        n = self.shape[0] * self.shape[1]
        return {s: float(self.leaf[s].sum() * s * s) / n for s in self.sizes}


@dataclass
class PermutedAllocation:
    """PermutedQTAllocation fields (mtc/core/permutation.py:54-67); ``dequant``
    is in the original channel order (permutation.py:76-79)."""
    inner: Allocation
    row_perm: np.ndarray
    col_perm: np.ndarray
    total_bits: int
    source: Optional[np.ndarray] = field(default=None, repr=False)
    _dequant: Optional[np.ndarray] = field(default=None, repr=False)

    @property
    def bits_per_element(self) -> float:
        K, N = self.inner.shape
        return self.total_bits / (K * N)

    @property
    def dequant(self) -> np.ndarray:
        if self._dequant is None:
            if self.source is None:
                raise ValueError("this allocation does not hold its matrix; use permuted_qt_dequant(W, ...)")
            self._dequant = _gpu_dequant(self.source, self)
        return self._dequant


def _gpu_dequant(W: np.ndarray, alloc) -> np.ndarray:
    from ..kernels.gemm import MTCMatrix

    return MTCMatrix.from_qt_allocation(np.asarray(W, np.float32), alloc).to_array()


def qt_dequant(W, sizes, leaf, modes, scales) -> np.ndarray:
    """Exact reconstruction of an MTC-QT allocation of W (the reference's
    qt_dequant, mtc/core/quadtree.py:157-171), computed by the GPU dequant
    kernel: q = clip(rint(w / s)) per leaf, then q * s in fp32."""
    W = np.asarray(W, np.float32)
    a = Allocation(tuple(int(s) for s in sizes), leaf, modes, scales, 0, W.shape)
    return _gpu_dequant(W, a)


def unpermute(Wp, row_perm, col_perm) -> np.ndarray:
    """W with W[ix_(pr, pc)] = Wp (mtc/core/permutation.py:70-73)."""
    Wp = np.asarray(Wp)
    out = np.empty_like(Wp)
    out[np.ix_(np.asarray(row_perm), np.asarray(col_perm))] = Wp
    return out


def permuted_qt_dequant(W, row_perm, col_perm, sizes, leaf, modes, scales) -> np.ndarray:
    """Exact reconstruction of an MTC-QT-P allocation in the original channel
    order (mtc/core/permutation.py:76-79), on the GPU."""
    W = np.asarray(W, np.float32)
    inner = Allocation(tuple(int(s) for s in sizes), leaf, modes, scales, 0, W.shape)
    return _gpu_dequant(W, PermutedAllocation(inner, np.asarray(row_perm), np.asarray(col_perm), 0))


class _Level:
    def __init__(self, D, S, R, modes, meta_bits):
        self.D, self.S, self.R, self.modes, self.meta_bits = D, S, R, modes, meta_bits


def _sum4(x: torch.Tensor) -> torch.Tensor:
    a, b = x.shape[0] // 2, x.shape[1] // 2
    return x.reshape(a, 2, b, 2).sum(dim=(1, 3))


def _up4(x: torch.Tensor) -> torch.Tensor:
    return x.repeat_interleave(2, dim=0).repeat_interleave(2, dim=1)


class QuadtreeRD:
    """MTC-QT on the GPU: candidate tables once, then cheap ``select(budget)``."""

    def __init__(self, W, importance=None, sizes: Sequence[int] = (32, 16, 8),
                 modes: Sequence[int] = DEFAULT_MODES, scale_format: str = "bf16", device=None):
        lib = _lib.load()
        self.device = torch.device(device if device is not None else "cuda")
        Wt = W if isinstance(W, torch.Tensor) else torch.from_numpy(np.ascontiguousarray(W, dtype=np.float32))
        self.W = Wt.to(self.device, torch.float32).contiguous()
        self.W_host = W if isinstance(W, np.ndarray) else None
        self.sizes = tuple(sorted(sizes, reverse=True))
        for a, b in zip(self.sizes, self.sizes[1:]):
            assert a == 2 * b, "quadtree levels must halve: e.g. (32, 16, 8)"
        K, N = self.W.shape
        self.shape = (int(K), int(N))
        assert K % self.sizes[0] == 0 and N % self.sizes[0] == 0
        h = np.ones(K, dtype=np.float64) if importance is None else np.asarray(importance, dtype=np.float64)
        h = h / max(h.mean(), 1e-30)
        h_dev = torch.from_numpy(h).to(self.device)
        st = torch.cuda.current_stream(self.device).cuda_stream
        self.modes = tuple(sorted(modes))
        self.levels: Dict[int, _Level] = {}
        for s in self.sizes:
            a, b = K // s, N // s
            D = torch.empty(len(self.modes), a, b, dtype=torch.float64, device=self.device)
            S = torch.zeros(len(self.modes), a, b, dtype=torch.float32, device=self.device)
            for i, m in enumerate(self.modes):
                if m == 0:
                    blk = self.W.double().reshape(a, s, b, s)
                    D[i] = torch.einsum("arbc,ar->ab", blk * blk, h_dev.reshape(a, s))
                    continue
                al = torch.from_numpy(alpha_grid(m)).to(self.device)
                _lib.check(lib.mtc_rd_search(self.W.data_ptr(), K, N, s, h_dev.data_ptr(), m, al.data_ptr(),
                                             al.numel(), 1 if scale_format == "bf16" else 0, D[i].data_ptr(),
                                             S[i].data_ptr(), st), "rd search")
            R = torch.tensor([m * s * s for m in self.modes], dtype=torch.float64, device=self.device)
            self.levels[s] = _Level(D, S, R, self.modes, META_BITS[scale_format])

    def _solve(self, lam: float):
        idx, leaf_J, leaf_R = {}, {}, {}
        for s, c in self.levels.items():
            rates = c.R[:, None, None] + c.meta_bits
            J = c.D + lam * rates
            i = torch.argmin(J, dim=0)
            idx[s] = i
            leaf_J[s] = torch.gather(J, 0, i[None])[0]
            leaf_R[s] = torch.gather(rates.expand_as(J), 0, i[None])[0]
        fine = self.sizes[-1]
        J, R = leaf_J[fine], leaf_R[fine]
        keep = {fine: torch.ones_like(J, dtype=torch.bool)}
        for s in reversed(self.sizes[:-1]):
            sJ, sR = _sum4(J), _sum4(R)
            k = leaf_J[s] <= sJ
            keep[s] = k
            J = torch.where(k, leaf_J[s], sJ) + lam * FLAG_BITS
            R = torch.where(k, leaf_R[s], sR) + FLAG_BITS
        return R, keep, idx

    def select(self, bits_per_element: float) -> Allocation:
        budget = bits_per_element * self.shape[0] * self.shape[1]
        Dmax = max(float(c.D.max()) for c in self.levels.values())
        scale_ref = max(Dmax, 1e-30) / (2 * self.sizes[-1] ** 2)
        # bisection on log(lambda) between scale_ref * 1e-16 and scale_ref * 1e6,
        # 60 halvings, keeping the cheapest solution that fits the budget
        # (the same bracket and step count as the reference, for identical
        # allocations: mtc/core/quadtree.py:126-140)
        log_lo, log_hi = np.log(scale_ref * 1e-16), np.log(scale_ref * 1e6)
        fit = self._solve(float(np.exp(log_hi)))
        if float(fit[0].sum()) > budget:
            raise ValueError(f"{bits_per_element} bits per element is below what this matrix needs "
                             f"({float(fit[0].sum()) / (self.shape[0] * self.shape[1]):.3f} at the coarsest "
                             f"allocation)")
        for _ in range(60):
            lam_log = 0.5 * (log_lo + log_hi)
            trial = self._solve(float(np.exp(lam_log)))
            if float(trial[0].sum()) <= budget:
                fit, log_hi = trial, lam_log
            else:
                log_lo = lam_log
        R, keep, idx = fit
        # a node is a leaf when every ancestor was split and it is kept
        reach = {self.sizes[0]: torch.ones_like(keep[self.sizes[0]])}
        leaf = {}
        for lvl, s in enumerate(self.sizes):
            leaf[s] = reach[s] & keep[s]
            if lvl + 1 < len(self.sizes):
                reach[self.sizes[lvl + 1]] = _up4(reach[s] & ~keep[s])
        modes, scales = {}, {}
        mode_tab = torch.tensor(self.modes, dtype=torch.uint8, device=self.device)
        for s in self.sizes:
            c = self.levels[s]
            mg = mode_tab[idx[s]]
            sg = torch.gather(c.S, 0, idx[s][None])[0]
            modes[s] = torch.where(leaf[s], mg, torch.zeros_like(mg)).cpu().numpy()
            scales[s] = torch.where(leaf[s], sg, torch.zeros_like(sg)).cpu().numpy()
        return Allocation(self.sizes, {s: leaf[s].cpu().numpy() for s in self.sizes}, modes, scales,
                          int(float(R.sum())), self.shape, source=self.W_host)


def channel_orders(W: np.ndarray, importance, rows=True, cols=True):
    """Stable ascending sort of each channel's weighted energy (permutation.py:34-46)."""
    K, N = W.shape
    h = np.ones(K) if importance is None else np.asarray(importance, dtype=np.float64)
    e = h[:, None] * (np.asarray(W, dtype=np.float64) ** 2)
    pr = np.argsort(e.sum(axis=1), kind="stable") if rows else np.arange(K)
    pc = np.argsort(e.sum(axis=0), kind="stable") if cols else np.arange(N)
    return pr, pc


def index_bits(K: int, N: int, rows: bool = True, cols: bool = True) -> int:
    return (K * ceil(log2(K)) if rows else 0) + (N * ceil(log2(N)) if cols else 0)


class PermutedQuadtreeRD:
    """MTC-QT-P on the GPU (channel sort on the host, MTC-QT on the device)."""

    def __init__(self, W, importance=None, sizes: Sequence[int] = (32, 16, 8),
                 modes: Sequence[int] = DEFAULT_MODES, scale_format: str = "bf16", rows=True, cols=True,
                 device=None):
        self.W = np.asarray(W, dtype=np.float32)
        h = None if importance is None else np.asarray(importance)
        self.pr, self.pc = channel_orders(self.W, h, rows, cols)
        self.perm_bits = index_bits(*self.W.shape, rows, cols)
        self.qt = QuadtreeRD(self.W[self.pr][:, self.pc], None if h is None else h[self.pr], sizes, modes,
                             scale_format, device)

    def select(self, bits_per_element: float) -> PermutedAllocation:
        inner = self.qt.select(bits_per_element - self.perm_bits / self.W.size)
        return PermutedAllocation(inner, self.pr, self.pc, inner.total_bits + self.perm_bits, source=self.W)


def qt_allocate(W, bits_per_element: float, importance=None, sizes: Sequence[int] = (32, 16, 8),
                modes: Sequence[int] = DEFAULT_MODES, device=None) -> Allocation:
    """One-call MTC-QT allocation (mtc/core/quadtree.py:174-181), on the GPU."""
    return QuadtreeRD(W, importance, sizes, modes, device=device).select(bits_per_element)
