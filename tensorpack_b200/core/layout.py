"""Reference-layout packing of MTC matrices and the leaf lists the GPU repack reads.

Host-side format logic only (numpy): turning an allocation (fixed-block or
quadtree) into integer codes and an arena with the reference's per-mode byte
packing, ordering leaves for the device stream, and bit accounting.  No GEMM
or dequantisation runs here; those are CUDA kernels.

Reference behaviour mirrored here:
  * code formula  q = clip(rint(w / s), lo, hi), s == 0 -> 1  (allocation.py:89-94)
  * payload  m * s * s / 8 bytes per leaf, codes row-major inside the leaf,
    LSB-first m-bit fields (P2 crumbs, P4 nibbles, P8 bytes, P16 little-endian,
    P3/5/6 bitstream)  (gemm.py:457-478, packing.py:12-45)
  * offsets  exclusive prefix sum of payload sizes in leaf order (gemm.py:449-454)
  * accounting  payload + per-leaf scale/mode metadata + one split flag per
    node above the finest level + permutation index bits
    (quadtree.py:97-117, permutation.py:49-51, allocation.py:197)
"""

from __future__ import annotations

from dataclasses import dataclass
from math import ceil, log2
from typing import Optional, Sequence, Tuple

import numpy as np

from .types import META_BITS, QRANGE, SPLIT_FLAG_BITS

TILE = 32          # device tile edge
MB = 4             # micro-block edge; smallest supported leaf
SUPPORTED_LEAF_SIZES = (4, 8, 16, 32)

# Mirrors `struct mtc_leaf_in` of include/mtc_b200.h (12 bytes).
LEAF_IN_DTYPE = np.dtype([("arena_off", "<u4"), ("scale_bits", "<u4"), ("mode", "u1"), ("z0", "u1"),
                          ("size", "u1"), ("pad_", "u1")])
assert LEAF_IN_DTYPE.itemsize == 12


def quantize_codes(blocks: np.ndarray, mode: int, scales: np.ndarray) -> np.ndarray:
    """Integer codes (as fp32) of blocks (..., s, s) with per-block scales (...)."""
    lo, hi = QRANGE[mode]
    s = np.asarray(scales, dtype=np.float32)[..., None, None]
    s = np.where(s == 0.0, np.float32(1.0), s)
    return np.clip(np.round(np.asarray(blocks, np.float32) / s), lo, hi)


def pack_bitstream(q: np.ndarray, m: int) -> np.ndarray:
    """Rows of signed integer codes -> rows of LSB-first m-bit payload bytes."""
    q = np.asarray(q, dtype=np.int64)
    u = (q & ((1 << m) - 1)).astype(np.uint32)
    bits = ((u[..., None] >> np.arange(m, dtype=np.uint32)) & 1).astype(np.uint8)
    return np.packbits(bits.reshape(q.shape[0], -1), axis=1, bitorder="little")


def z_index(i, j):
    """Z-order index of micro-block (i, j) inside a 32x32 tile (i, j in 0..7)."""
    i = np.asarray(i)
    j = np.asarray(j)
    return (((i >> 2) & 1) << 5 | ((j >> 2) & 1) << 4 | ((i >> 1) & 1) << 3 | ((j >> 1) & 1) << 2
            | (i & 1) << 1 | (j & 1))


def bf16_exact(x: np.ndarray) -> bool:
    b = np.asarray(x, dtype=np.float32).view(np.uint32)
    return bool(np.all((b & 0xFFFF) == 0))


@dataclass
class LeafSet:
    """Leaves of a packed matrix: top-left (row, col), edge, mode, scale and
    the byte offset of the payload in the arena.  Coordinates are in the
    stored (possibly permuted) matrix."""

    row: np.ndarray
    col: np.ndarray
    size: np.ndarray
    mode: np.ndarray
    scale: np.ndarray
    offset: np.ndarray

    def __len__(self):
        return int(self.row.shape[0])

    def take(self, idx) -> "LeafSet":
        return LeafSet(self.row[idx], self.col[idx], self.size[idx], self.mode[idx], self.scale[idx],
                       self.offset[idx])

    @property
    def payload_bytes(self) -> np.ndarray:
        return (self.mode.astype(np.int64) * self.size.astype(np.int64) ** 2) // 8


def canonical_order(ls: LeafSet) -> np.ndarray:
    """Tile-major (32x32 tiles in row-major order), Z order inside a tile."""
    tr, tc = ls.row // TILE, ls.col // TILE
    z = z_index((ls.row % TILE) // MB, (ls.col % TILE) // MB)
    ntc = int(tc.max()) + 1 if len(ls) else 1
    return np.lexsort((z, tr * ntc + tc))


def leaves_from_grid(modes: np.ndarray, scales: np.ndarray, block_size: int,
                     offsets: Optional[np.ndarray] = None) -> LeafSet:
    """Fixed-block allocation grid (row-major block order) as a leaf set."""
    a, b = modes.shape
    ii, jj = np.meshgrid(np.arange(a), np.arange(b), indexing="ij")
    n = a * b
    return LeafSet(
        row=(ii.ravel() * block_size).astype(np.int64),
        col=(jj.ravel() * block_size).astype(np.int64),
        size=np.full(n, block_size, dtype=np.int64),
        mode=np.asarray(modes, dtype=np.uint8).ravel().copy(),
        scale=np.asarray(scales, dtype=np.float32).ravel().copy(),
        offset=(np.zeros(n, np.int64) if offsets is None else np.asarray(offsets, np.int64).ravel().copy()),
    )


def leaves_from_quadtree(sizes: Sequence[int], leaf: dict, modes: dict, scales: dict) -> LeafSet:
    """Leaves of a quadtree allocation (QTAllocation fields, quadtree.py:55-61),
    in canonical order with offsets not yet assigned."""
    rows, cols, sz, md, sc = [], [], [], [], []
    for s in sizes:
        ii, jj = np.nonzero(leaf[s])
        rows.append(ii.astype(np.int64) * s)
        cols.append(jj.astype(np.int64) * s)
        sz.append(np.full(ii.shape[0], s, dtype=np.int64))
        md.append(np.asarray(modes[s])[ii, jj].astype(np.uint8))
        sc.append(np.asarray(scales[s])[ii, jj].astype(np.float32))
    ls = LeafSet(np.concatenate(rows), np.concatenate(cols), np.concatenate(sz), np.concatenate(md),
                 np.concatenate(sc), np.zeros(sum(len(r) for r in rows), np.int64))
    return ls.take(canonical_order(ls))


def leaf_codes(W: np.ndarray, ls: LeafSet, idx: np.ndarray, s: int, m: int) -> np.ndarray:
    """Codes (n, s*s) of leaves `idx` (all of edge s and mode m) of matrix W."""
    r = ls.row[idx][:, None, None] + np.arange(s)[None, :, None]
    c = ls.col[idx][:, None, None] + np.arange(s)[None, None, :]
    blocks = np.asarray(W, dtype=np.float32)[r, c]
    return quantize_codes(blocks, m, ls.scale[idx]).reshape(len(idx), s * s).astype(np.int64)


def pack_leaves(W: np.ndarray, ls: LeafSet, codes: Optional[np.ndarray] = None) -> Tuple[np.ndarray, np.ndarray]:
    """Arena bytes and per-leaf offsets (leaf order = payload order).

    ``codes`` optionally gives explicit integer codes for every element of the
    stored matrix (e.g. GPTQ output); they must lie in each leaf's range."""
    nbytes = ls.payload_bytes
    offsets = np.concatenate([[0], np.cumsum(nbytes)[:-1]]).astype(np.int64) if len(ls) else np.zeros(0, np.int64)
    total = int(nbytes.sum())
    arena = np.zeros(max(total, 1), dtype=np.uint8)
    for s in np.unique(ls.size):
        for m in np.unique(ls.mode[ls.size == s]):
            m = int(m)
            if m == 0:
                continue
            idx = np.nonzero((ls.size == s) & (ls.mode == m))[0]
            if codes is None:
                q = leaf_codes(W, ls, idx, int(s), m)
            else:
                r = ls.row[idx][:, None, None] + np.arange(s)[None, :, None]
                c = ls.col[idx][:, None, None] + np.arange(s)[None, None, :]
                q = np.asarray(codes)[r, c].reshape(len(idx), int(s) * int(s)).astype(np.int64)
                lo, hi = QRANGE[m]
                if q.min() < lo or q.max() > hi:
                    raise ValueError(f"explicit codes outside the P{m} range [{lo}, {hi}]")
            packed = pack_bitstream(q, m)
            dest = offsets[idx][:, None] + np.arange(packed.shape[1])
            arena[dest] = packed
    return arena, offsets


def flag_bits(ls: LeafSet, sizes: Sequence[int]) -> int:
    """Split-flag bits of a quadtree: one per reached node above the finest
    level (leaves there, plus every ancestor of a smaller leaf)."""
    sizes = tuple(sorted(sizes, reverse=True))
    total = 0
    for s in sizes[:-1]:
        n_leaf = int((ls.size == s).sum())
        small = ls.size < s
        anc = np.unique((ls.row[small] // s) * (1 << 32) + ls.col[small] // s)
        total += (n_leaf + anc.shape[0]) * SPLIT_FLAG_BITS
    return total


def index_bits(K: int, N: int, rows: bool, cols: bool) -> int:
    """Bits of stored permutations (permutation.py:49-51)."""
    return (K * ceil(log2(K)) if rows else 0) + (N * ceil(log2(N)) if cols else 0)


def padded_leaves(ls: LeafSet, K: int, N: int) -> LeafSet:
    """Add P0 4x4 leaves covering the padding up to multiples of 32."""
    Kp, Np = -(-K // TILE) * TILE, -(-N // TILE) * TILE
    if Kp == K and Np == N:
        return ls
    if K % MB or N % MB:
        raise ValueError(f"shape ({K}, {N}) must be a multiple of {MB}")
    ii, jj = np.meshgrid(np.arange(Kp // MB), np.arange(Np // MB), indexing="ij")
    pad = (ii * MB >= K) | (jj * MB >= N)
    r = (ii[pad] * MB).astype(np.int64)
    c = (jj[pad] * MB).astype(np.int64)
    n = r.shape[0]
    extra = LeafSet(r, c, np.full(n, MB, np.int64), np.zeros(n, np.uint8), np.zeros(n, np.float32),
                    np.zeros(n, np.int64))
    return LeafSet(*(np.concatenate([getattr(ls, f), getattr(extra, f)])
                     for f in ("row", "col", "size", "mode", "scale", "offset")))


def device_leaf_list(ls: LeafSet, K: int, N: int):
    """(leaf_in structured array, tile CSR [T+1] uint32, tk, tn) for the repack."""
    for s in np.unique(ls.size):
        if int(s) not in SUPPORTED_LEAF_SIZES:
            raise ValueError(f"leaf edge {int(s)} not supported on the device (edges 4, 8, 16, 32)")
    full = padded_leaves(ls, K, N)
    order = canonical_order(full)
    full = full.take(order)
    tk, tn = -(-K // TILE), -(-N // TILE)
    tile = (full.row // TILE) * tn + full.col // TILE
    counts = np.bincount(tile, minlength=tk * tn)
    begin = np.zeros(tk * tn + 1, dtype=np.uint32)
    np.cumsum(counts, out=begin[1:])
    out = np.zeros(len(full), dtype=LEAF_IN_DTYPE)
    out["arena_off"] = full.offset.astype(np.uint32)
    out["scale_bits"] = np.where(full.mode == 0, np.float32(0), full.scale).astype(np.float32).view(np.uint32)
    out["mode"] = full.mode
    out["z0"] = z_index((full.row % TILE) // MB, (full.col % TILE) // MB).astype(np.uint8)
    out["size"] = full.size.astype(np.uint8)
    return out, begin, tk, tn


def choose_exp2(ls: LeafSet) -> int:
    """Power-of-two pre-scale so the largest |q * s| of any leaf maps to at
    most 2^15 in the fp16 tensor path."""
    live = ls.mode != 0
    if not live.any():
        return 0
    qmax = np.ldexp(1.0, ls.mode[live].astype(np.int64) - 1)
    bound = float(np.max(np.abs(ls.scale[live].astype(np.float64)) * qmax))
    if bound <= 0.0 or not np.isfinite(bound):
        return 0
    return int(max(-60, min(60, 15 - ceil(log2(bound)))))
