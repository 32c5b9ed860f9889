"""Permutation folding and the fused epilogue's host side (CPU only).

The composition rule of tensorpack_b200.kernels.fold is checked with the
oracle standing in for the kernels: layer A (MTC-QT-P) leaves its output in
stored column order, B's input permutation absorbs A's column permutation,
and the chain must equal act(X @ Wa + ba) @ Wb + bb computed in original
order.  Also: argument checks of the epilogue and of the folding helpers.
"""

import numpy as np
import pytest

import inputs
from oracle import mtc_oracle as O
from tensorpack_b200.kernels.fold import fold_permutation, inverse_permutation, with_permutations
from tensorpack_b200.kernels.gemm import MTCMatrix
from test_host_layout import decode_arena

ACTS = {
    None: lambda y: y,
    "relu": lambda y: np.maximum(y, 0.0),
    "silu": lambda y: y / (1.0 + np.exp(-y)),
}


def _permuted(K, N, seed):
    W, sizes, leaf, modes, scales = inputs.forced_mode_allocation(K, N, seed=seed, p_split=0.5)
    rng = np.random.default_rng(seed + 100)
    pr, pc = rng.permutation(K), rng.permutation(N)
    inner = O.QuadtreeAllocation(sizes, leaf, modes, scales, None, 0)
    m = MTCMatrix.from_qt_allocation(W, O.PermutedAllocation(inner, pr, pc, None, 0))
    return m, O.permuted_quadtree_dequant(W, pr, pc, sizes, leaf, modes, scales).astype(np.float64)


def _apply(mat: MTCMatrix, X, bias, act):
    """What the kernels compute for one layer, with the oracle's exact stored
    matrix: Y[:, pc] = act(X[:, pr] @ Wp + bias[pc]) (bias in Y's order)."""
    Wp = decode_arena(mat).astype(np.float64)
    Xg = X if mat.row_perm is None else X[:, mat.row_perm]
    Yp = Xg @ Wp
    if mat.col_perm is None:
        return ACTS[act](Yp + bias)
    Y = np.empty_like(Yp)
    Y[:, mat.col_perm] = Yp
    return ACTS[act](Y + bias)


@pytest.mark.parametrize("act", [None, "relu", "silu"])
@pytest.mark.parametrize("b_permuted", [True, False])
def test_folded_chain_equals_original(act, b_permuted):
    A, WA = _permuted(64, 96, seed=3)
    B, WB = _permuted(96, 128, seed=4)
    if not b_permuted:
        B = with_permutations(B, None, B.col_perm)
        WB = np.empty((96, 128))
        WB[:, B.col_perm] = decode_arena(B)
    rng = np.random.default_rng(9)
    X = rng.standard_normal((5, 64))
    ba, bb = rng.standard_normal(96), rng.standard_normal(128)
    ref = ACTS[act](X @ WA + ba) @ WB + bb
    A2, B2 = fold_permutation(A, B)
    assert A2.col_perm is None and A2.row_perm is not None
    np.testing.assert_array_equal(A2.row_perm, A.row_perm)
    mid = _apply(A2, X, ba[A.col_perm], act)            # stored column order
    out = _apply(B2, mid, bb, None)
    np.testing.assert_allclose(out, ref, rtol=1e-10, atol=1e-9)
    # the unfolded chain, for comparison
    np.testing.assert_allclose(_apply(B, _apply(A, X, ba, act), bb, None), ref, rtol=1e-10, atol=1e-9)


def test_folding_shares_the_packed_layout():
    A, _ = _permuted(64, 96, seed=5)
    B, _ = _permuted(96, 64, seed=6)
    A2, B2 = fold_permutation(A, B)
    assert A2.arena is A.arena and B2.arena is B.arena
    assert np.array_equal(B2.row_perm, inverse_permutation(A.col_perm)[B.row_perm])
    # nothing to fold when A has no column permutation
    A3 = with_permutations(A, A.row_perm, None)
    assert fold_permutation(A3, B) == (A3, B)
    with pytest.raises(ValueError, match="chain"):
        fold_permutation(A, A)
    with pytest.raises(ValueError, match="permutation"):
        with_permutations(A, np.zeros(64, np.int64), None)


def test_epilogue_arguments():
    import torch

    from tensorpack_b200 import _lib
    from tensorpack_b200.kernels.device import epilogue
    from tensorpack_b200.nn.layers import LinearMTCAdaptive

    assert epilogue(None, None) is None
    e = epilogue(None, "silu")
    assert e.act == _lib.ACT_SILU and not e.bias
    with pytest.raises(ValueError, match="activation"):
        epilogue(None, "tanh")
    with pytest.raises(ValueError, match="CUDA"):
        epilogue(torch.zeros(4), None)
    with pytest.raises(ValueError, match="activation"):
        LinearMTCAdaptive(32, 16, activation="swish")


def test_layer_numpy_forward_applies_activation_after_bias():
    """The numpy forward path's activation formulas (the GPU path fuses the
    same functions); checked here without a GPU on the host-side helpers."""
    from tensorpack_b200.nn.layers import _NP_ACT

    y = np.array([-3.0, -0.5, 0.0, 0.5, 3.0], np.float32)
    np.testing.assert_array_equal(_NP_ACT["relu"](y), np.array([0, 0, 0, 0.5, 3], np.float32))
    np.testing.assert_allclose(_NP_ACT["silu"](y), y / (1 + np.exp(-y.astype(np.float64))), rtol=1e-6)
    g = 0.5 * y * (1 + np.tanh(np.sqrt(2 / np.pi) * (y + 0.044715 * y.astype(np.float64) ** 3)))
    np.testing.assert_allclose(_NP_ACT["gelu_tanh"](y), g, rtol=1e-6, atol=1e-7)
