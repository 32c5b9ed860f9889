"""Host-side format tests (CPU only): reference-layout packing, quadtree leaf
ordering, bit accounting and the leaf list handed to the GPU repack."""

import os

import numpy as np
import pytest

import inputs
from oracle import mtc_oracle as O
from tensorpack_b200.core import layout
from tensorpack_b200.kernels.gemm import MTCMatrix


def load(golden_dir, name):
    return np.load(os.path.join(golden_dir, name))


def qt_from_golden(g, prefix):
    sizes = tuple(int(s) for s in g[prefix + "sizes"])
    leaf = {s: g[f"{prefix}leaf_{s}"] for s in sizes}
    modes = {s: g[f"{prefix}modes_{s}"] for s in sizes}
    scales = {s: g[f"{prefix}scales_{s}"] for s in sizes}
    return O.QuadtreeAllocation(sizes, leaf, modes, scales, None, int(g[prefix + "total_bits"]))


def decode_arena(m: MTCMatrix) -> np.ndarray:
    """Oracle decode of every leaf payload of a packed matrix (stored order)."""
    ls = m.leaf_set
    K, N = m.shape
    out = np.zeros((K, N), np.float32)
    for i in range(len(ls)):
        md, s = int(ls.mode[i]), int(ls.size[i])
        if md == 0:
            continue
        q = O.bitstream_unpack(m.arena.raw_buffer, int(ls.offset[i]), s * s, md).reshape(s, s)
        out[ls.row[i]:ls.row[i] + s, ls.col[i]:ls.col[i] + s] = q.astype(np.float32) * np.float32(ls.scale[i])
    return out + np.float32(0.0)


@pytest.mark.parametrize("b", [2.6, 5.2, 9.0])
def test_from_allocation_matches_reference_arena(golden_dir, b):
    g = load(golden_dir, "fixed_pair.npz")
    A, B = inputs.fixed_pair(seed=5)
    tag = f"b{b}_"
    for nm, X in (("A", A), ("B", B)):
        m = MTCMatrix.from_allocation(X, g[tag + nm + "_modes"], g[tag + nm + "_scales"], 16)
        n = int(g[tag + nm + "_payload_bits"]) // 8
        assert m.total_bytes_allocated == n
        np.testing.assert_array_equal(m.arena.raw_buffer[:n], g[tag + nm + "_arena"])
        np.testing.assert_array_equal(m.offsets, g[tag + nm + "_offsets"])
        np.testing.assert_array_equal(decode_arena(m), g[tag + nm + "_dequant"])


@pytest.mark.parametrize("tag", ["layer", "heavy"])
def test_from_numpy_matches_reference(golden_dir, tag):
    g = load(golden_dir, "legacy_from_numpy.npz")
    W = inputs.linear_fp32_weight(32, 16, seed=42) if tag == "layer" else inputs.heavy_tailed(64, 64, seed=9)
    m = MTCMatrix.from_numpy(W, block_size=16, epsilon=0.05, use_pointer_hierarchy=False)
    np.testing.assert_array_equal(m.precisions, g[tag + "_precisions"])
    np.testing.assert_array_equal(m.scales, g[tag + "_scales"])
    np.testing.assert_array_equal(m.offsets, g[tag + "_offsets"])
    np.testing.assert_array_equal(m.arena.raw_buffer[:m.total_bytes_allocated], g[tag + "_arena"])
    np.testing.assert_array_equal(decode_arena(m), g[tag + "_dequant"])


@pytest.mark.parametrize("b", [2.0, 3.0, 4.5, 7.0])
def test_quadtree_pack_and_accounting(golden_dir, b):
    g = load(golden_dir, "qt_outlier_128.npz")
    W = inputs.outlier_matrix(128, seed=0)
    a = qt_from_golden(g, f"b{b}_")
    m = MTCMatrix.from_qt_allocation(W, a)
    assert m.is_quadtree and m.row_perm is None
    np.testing.assert_array_equal(decode_arena(m), g[f"b{b}_dequant"])
    assert m.accounted_bits == a.total_bits
    # payload bytes in the arena == payload bits of the allocation
    ls = m.leaf_set
    assert m.total_bytes_allocated * 8 == int((ls.mode.astype(np.int64) * ls.size ** 2).sum())


@pytest.mark.parametrize("sizes", [(32, 16, 8), (32, 16, 8, 4)])
def test_permuted_quadtree_pack_and_accounting(golden_dir, sizes):
    g = load(golden_dir, "qtp_rows_256.npz")
    W, _ = inputs.row_scaled(256, 256, seed=0)
    tag = f"s{len(sizes)}_"
    inner = qt_from_golden(g, tag + "inner_")
    alloc = O.PermutedAllocation(inner, g[tag + "row_perm"], g[tag + "col_perm"], None, int(g[tag + "total_bits"]))
    m = MTCMatrix.from_qt_allocation(W, alloc)
    stored = decode_arena(m)
    np.testing.assert_array_equal(O.unpermute(stored, m.row_perm, m.col_perm), g[tag + "dequant"])
    assert m.accounted_bits == alloc.total_bits


def test_leaf_order_is_tile_major_z_order(golden_dir):
    g = load(golden_dir, "qt_outlier_128.npz")
    m = MTCMatrix.from_qt_allocation(inputs.outlier_matrix(128, seed=0), qt_from_golden(g, "b3.0_"))
    leaves, begin, tk, tn = layout.device_leaf_list(m.leaf_set, 128, 128)
    assert (tk, tn) == (4, 4) and begin[-1] == len(leaves)
    for t in range(tk * tn):
        lv = leaves[begin[t]:begin[t + 1]]
        zrun = 0
        for L in lv:  # contiguous, aligned Z ranges that cover all 64 micro-blocks
            nmb = (int(L["size"]) // 4) ** 2
            assert int(L["z0"]) == zrun and zrun % nmb == 0
            zrun += nmb
        assert zrun == 64


def test_ragged_shape_gets_p0_padding():
    """K, N not multiples of 32 (root 16): the leaf list is padded with P0 4x4 leaves."""
    rng = np.random.default_rng(1)
    W = rng.standard_normal((48, 80)).astype(np.float32)
    modes = rng.choice([0, 2, 3, 4, 8], size=(3, 5)).astype(np.uint8)
    scales = (np.abs(W.reshape(3, 16, 5, 16)).max(axis=(1, 3)) / 7).astype(np.float32)
    m = MTCMatrix.from_allocation(W, modes, scales, 16)
    leaves, begin, tk, tn = layout.device_leaf_list(m.leaf_set, 48, 80)
    assert (tk, tn) == (2, 3)
    n_pad = int(((leaves["mode"] == 0) & (leaves["size"] == 4)).sum())
    assert n_pad == (64 * 96 - 48 * 80) // 16
    for t in range(tk * tn):
        lv = leaves[begin[t]:begin[t + 1]]
        assert sum((int(x) // 4) ** 2 for x in lv["size"]) == 64


def test_exp2_keeps_fp16_range():
    ls = layout.LeafSet(np.zeros(3, np.int64), np.zeros(3, np.int64), np.full(3, 4, np.int64),
                        np.array([4, 16, 2], np.uint8), np.array([1e-3, -2e-5, 7.0], np.float32), np.zeros(3, np.int64))
    e = layout.choose_exp2(ls)
    bound = max(1e-3 * 8, 2e-5 * 32768, 7.0 * 2)
    assert bound * 2.0 ** e <= 2 ** 15 < bound * 2.0 ** (e + 1)


def test_explicit_codes_must_fit_mode(golden_dir):
    g = load(golden_dir, "qt_outlier_128.npz")
    a = qt_from_golden(g, "b3.0_")
    W = inputs.outlier_matrix(128, seed=0)
    codes = np.zeros(W.shape, np.int64)
    m = MTCMatrix.from_qt_allocation(W, a, codes=codes)
    assert not decode_arena(m).any()
    codes[:] = 40000
    with pytest.raises(ValueError):
        MTCMatrix.from_qt_allocation(W, a, codes=codes)


def test_unsupported_level_rejected():
    a = O.QuadtreeAllocation((64, 32), {64: np.ones((1, 1), bool), 32: np.zeros((2, 2), bool)},
                             {64: np.full((1, 1), 4, np.uint8), 32: np.zeros((2, 2), np.uint8)},
                             {64: np.ones((1, 1), np.float32), 32: np.zeros((2, 2), np.float32)}, None, 0)
    with pytest.raises(ValueError):
        MTCMatrix.from_qt_allocation(np.zeros((64, 64), np.float32), a)


def gptq_fixture(golden_dir):
    """GPTQ codes on an MTC-QT-P grid, made by the reference
    (tests/golden/make_gptq_fixture.py): allocation, stored-order codes and
    the SHA-256 of the reference's dequantised GPTQ result."""
    g = load(golden_dir, "gptq_qtp_256.npz")
    sizes = tuple(int(s) for s in g["sizes"])
    inner = O.QuadtreeAllocation(sizes, {s: g[f"leaf_{s}"] for s in sizes}, {s: g[f"modes_{s}"] for s in sizes},
                                 {s: g[f"scales_{s}"] for s in sizes}, None, 0)
    a = O.PermutedAllocation(inner, g["row_perm"], g["col_perm"], None, int(g["total_bits"]))
    W, X = inputs.gptq_layer(256, 256, seed=0)
    return g, a, W, X


def test_gptq_codes_pack_to_the_reference_result(golden_dir):
    """Explicit (non-RTN) codes are packed as given: decoding the arena and
    undoing the permutation reproduces the reference's GPTQ output bit for
    bit (mtc/baselines/gptq.py:39-138 inside qt_element_grid)."""
    import hashlib

    g, a, W, _ = gptq_fixture(golden_dir)
    assert int(g["codes_differ_from_rtn"]) > 1000
    m = MTCMatrix.from_qt_allocation(W, a, codes=g["codes_stored"])
    Q = O.unpermute(decode_arena(m), g["row_perm"], g["col_perm"])
    assert hashlib.sha256(np.ascontiguousarray(Q).tobytes()).hexdigest() == str(g["Q_sha"])
    # the RTN packing of the same grid is a different matrix
    rtn = O.unpermute(decode_arena(MTCMatrix.from_qt_allocation(W, a)), g["row_perm"], g["col_perm"])
    assert not np.array_equal(rtn, Q)
