"""Pin the CPU oracle against vectors produced by the reference implementation.

The fixtures in tests/golden/ were written by tests/golden/make_golden.py from
the reference sources; the inputs are regenerated here from the same seeds.
Every comparison is exact (bit-for-bit) except the packed GEMM, which the
reference itself only pins to rel. error < 1e-5 (tests/test_allocation.py:83).
"""

import hashlib
import os

import numpy as np
import pytest

import inputs
from oracle import mtc_oracle as O


def load(golden_dir, name):
    return np.load(os.path.join(golden_dir, name))


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def assert_qt_equal(prefix, g, a):
    sizes = tuple(int(s) for s in g[prefix + "sizes"])
    assert tuple(a.sizes) == sizes
    for s in sizes:
        np.testing.assert_array_equal(a.leaf[s], g[f"{prefix}leaf_{s}"])
        np.testing.assert_array_equal(a.modes[s], g[f"{prefix}modes_{s}"])
        np.testing.assert_array_equal(a.scales[s], g[f"{prefix}scales_{s}"])
    assert a.total_bits == int(g[prefix + "total_bits"])
    assert sha(a.dequant) == str(g[prefix + "dequant_sha"])


def test_quadtree_outlier_candidates_and_budgets(golden_dir):
    g = load(golden_dir, "qt_outlier_128.npz")
    W = inputs.outlier_matrix(128, seed=0)
    qt = O.Quadtree(W, None, (32, 16, 8, 4))
    for s in (32, 16, 8, 4):
        np.testing.assert_array_equal(qt.cands[s].S, g[f"cand_S_{s}"])
        np.testing.assert_array_equal(qt.cands[s].D, g[f"cand_D_{s}"])
    for b in (2.0, 3.0, 4.5, 7.0):
        a = qt.select(b)
        assert_qt_equal(f"b{b}_", g, a)
        np.testing.assert_array_equal(a.dequant, g[f"b{b}_dequant"])
        # exact single coverage of the matrix by the leaves (tests/test_quadtree.py:24-34)
        cover = sum(np.kron(a.leaf[s].astype(int), np.ones((s, s), int)) for s in a.sizes)
        assert (cover == 1).all()
        assert a.bits_per_element <= b + 1e-9


@pytest.mark.parametrize("sizes,b", [((32, 16, 8), 3.0), ((32, 16, 8, 4), 4.25)])
def test_permuted_quadtree(golden_dir, sizes, b):
    g = load(golden_dir, "qtp_rows_256.npz")
    W, h = inputs.row_scaled(256, 256, seed=0)
    a = O.PermutedQuadtree(W, h, sizes).select(b)
    tag = f"s{len(sizes)}_"
    np.testing.assert_array_equal(a.row_perm, g[tag + "row_perm"])
    np.testing.assert_array_equal(a.col_perm, g[tag + "col_perm"])
    assert_qt_equal(tag + "inner_", g, a.inner)
    assert a.total_bits == int(g[tag + "total_bits"])
    np.testing.assert_array_equal(a.dequant, g[tag + "dequant"])
    rebuilt = O.permuted_quadtree_dequant(W, a.row_perm, a.col_perm, a.inner.sizes, a.inner.leaf,
                                          a.inner.modes, a.inner.scales)
    np.testing.assert_array_equal(rebuilt, a.dequant)
    assert a.total_bits == a.inner.total_bits + O.index_bits(256, 256)


@pytest.mark.parametrize("b", [3.125, 4.25])
def test_llm_like_permuted(golden_dir, b):
    g = load(golden_dir, "llm_like_256x512.npz")
    W, h = inputs.llm_like(256, 512, seed=1)
    a = O.PermutedQuadtree(W, h, (32, 16, 8, 4)).select(b)
    tag = f"b{b}_"
    np.testing.assert_array_equal(a.row_perm, g[tag + "row_perm"])
    np.testing.assert_array_equal(a.col_perm, g[tag + "col_perm"])
    assert_qt_equal(tag + "inner_", g, a.inner)
    assert a.total_bits == int(g[tag + "total_bits"])
    assert sha(a.dequant) == str(g[tag + "dequant_sha"])


def test_multiscale(golden_dir):
    g = load(golden_dir, "multiscale_256.npz")
    a = O.Quadtree(inputs.multiscale(256, seed=2), None, (32, 16, 8, 4)).select(2.5)
    assert_qt_equal("", g, a)


def test_cpu_ref_config(golden_dir):
    g = load(golden_dir, "cpu_ref_1024.npz")
    W, h, _ = inputs.cpu_ref_config()
    a = O.Quadtree(W, h, (32, 16, 8, 4)).select(3.125)
    assert_qt_equal("", g, a)


@pytest.mark.parametrize("b", [2.6, 5.2, 9.0])
def test_fixed_pair_packing_and_gemm(golden_dir, b):
    g = load(golden_dir, "fixed_pair.npz")
    A, B = inputs.fixed_pair(seed=5)
    # rd_allocate_pair (allocation.py:329-356): importance from the other operand
    hB = (A.astype(np.float64) ** 2).sum(axis=0)
    hA = (B.astype(np.float64) ** 2).sum(axis=1)
    ab = O.allocate_fixed(B, b, hB, 16)
    at = O.allocate_fixed(A.T, b, hA, 16)
    tag = f"b{b}_"
    np.testing.assert_array_equal(at.modes.T, g[tag + "A_modes"])
    np.testing.assert_array_equal(at.scales.T, g[tag + "A_scales"])
    np.testing.assert_array_equal(at.dequant.T, g[tag + "A_dequant"])
    np.testing.assert_array_equal(ab.modes, g[tag + "B_modes"])
    np.testing.assert_array_equal(ab.scales, g[tag + "B_scales"])
    np.testing.assert_array_equal(ab.dequant, g[tag + "B_dequant"])
    Ap = O.PackedFixed.from_allocation(A, g[tag + "A_modes"], g[tag + "A_scales"], 16)
    Bp = O.PackedFixed.from_allocation(B, g[tag + "B_modes"], g[tag + "B_scales"], 16)
    for nm, p in (("A", Ap), ("B", Bp)):
        n = int(g[tag + nm + "_payload_bits"]) // 8
        np.testing.assert_array_equal(p.arena[:n], g[tag + nm + "_arena"])
        np.testing.assert_array_equal(p.offsets, g[tag + nm + "_offsets"])
        np.testing.assert_array_equal(p.to_array(), g[tag + nm + "_dequant"])
    C = O.packed_gemm(Ap, Bp)
    assert O.relative_frobenius_error(g[tag + "gemm"], C) < 1e-5
    C_sim = g[tag + "A_dequant"].astype(np.float64) @ g[tag + "B_dequant"]
    assert O.relative_frobenius_error(C_sim, C) < 1e-5


def test_fixed_bf16_with_importance(golden_dir):
    g = load(golden_dir, "fixed_bf16_256.npz")
    W, h = inputs.llm_like(256, 256, seed=3)
    c = O.candidates(W, h, 16, scale_format="bf16")
    np.testing.assert_array_equal(c.S, g["cand_S"])
    np.testing.assert_array_equal(c.D, g["cand_D"])
    al = O.select_fixed(c, 3.125)
    np.testing.assert_array_equal(al.modes, g["modes"])
    np.testing.assert_array_equal(al.scales, g["scales"])
    np.testing.assert_array_equal(al.dequant, g["dequant"])
    assert al.payload_bits == int(g["payload_bits"]) and al.meta_bits == int(g["meta_bits"])
    np.testing.assert_array_equal(O.fixed_dequant(W, al.modes, al.scales, 16), g["dequant"])


def test_bitstream_roundtrip_all_modes():
    rng = np.random.default_rng(0)
    for m, (lo, hi) in O.QRANGE.items():
        q = rng.integers(lo, hi + 1, size=(5, 64))
        packed = O.bitstream_pack(q, m)
        assert packed.shape[1] == 64 * m // 8
        for r in range(5):
            np.testing.assert_array_equal(O.bitstream_unpack(packed[r], 0, 64, m), q[r])
