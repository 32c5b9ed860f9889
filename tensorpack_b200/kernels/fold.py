"""Permutation folding between neighbouring layers.

An MTC-QT-P layer computes Y[:, pc] = X[:, pr] @ Wp (mtc/core/permutation.py:
15-21): an O(M K) gather before the product and an O(M N) scatter after it
(the reference lists folding them into neighbours as future work,
README.md:114).  When layer A feeds layer B through column-wise operations
only (bias, activation), A's scatter and B's gather compose into one
permutation: A' leaves its output in stored column order (no scatter) and B'
gathers its input through

    pr_B' = inv(pc_A)[pr_B]          (pr_B = identity when B is unpermuted)

because Y_A[:, j] = Yp_A[:, inv(pc_A)[j]].  B's gather is the fp16
conversion pass its kernel runs anyway, so the folded chain does one pass
over the activations fewer; A's bias, kept in original order by the caller,
is permuted to A's stored order.  The packed weights and device streams are
shared; nothing is repacked.
"""

from __future__ import annotations

from typing import Optional, Tuple

import numpy as np

from .gemm import MTCMatrix


def inverse_permutation(p: np.ndarray) -> np.ndarray:
    p = np.asarray(p, dtype=np.int64)
    inv = np.empty_like(p)
    inv[p] = np.arange(p.shape[0], dtype=np.int64)
    return inv


def with_permutations(mat: MTCMatrix, row_perm: Optional[np.ndarray], col_perm: Optional[np.ndarray]) -> MTCMatrix:
    """A matrix sharing ``mat``'s packed layout (and its device streams) with
    other row / column permutations."""
    K, N = mat.shape
    for p, n, what in ((row_perm, K, "row"), (col_perm, N, "column")):
        if p is not None and not np.array_equal(np.sort(np.asarray(p)), np.arange(n)):
            raise ValueError(f"{what} permutation is not a permutation of {n}")
    out = MTCMatrix(mat.shape, mat.block_size, mat.arena, mat.offsets, mat.precisions, mat.scales,
                    mat.pointer_tensor, leaf_rows=mat.leaf_rows, leaf_cols=mat.leaf_cols, leaf_sizes=mat.leaf_sizes,
                    sizes=mat.sizes if mat.is_quadtree else None, row_perm=row_perm, col_perm=col_perm)
    for ds in mat._device.values():
        out.attach_device_stream(ds.with_perms(out.row_perm, out.col_perm))
    return out


def fold_permutation(prev: MTCMatrix, nxt: MTCMatrix) -> Tuple[MTCMatrix, MTCMatrix]:
    """(prev', nxt'): prev' writes its output in stored column order and nxt'
    reads that order, so nxt'(act(prev'(X))) == nxt(act(prev(X))) for any
    column-wise act, with the scatter of prev and the separate gather of nxt
    folded into nxt's input permutation."""
    if prev.shape[1] != nxt.shape[0]:
        raise ValueError(f"shapes do not chain: {prev.shape} then {nxt.shape}")
    if prev.col_perm is None:
        return prev, nxt
    inv = inverse_permutation(prev.col_perm)
    pr = inv if nxt.row_perm is None else inv[np.asarray(nxt.row_perm, dtype=np.int64)]
    return (with_permutations(prev, prev.row_perm, None), with_permutations(nxt, pr, nxt.col_perm))
