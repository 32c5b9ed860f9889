"""GPU allocator (mtc_rd_search + tensor-op pruning) against the reference.

The scale search must reproduce the reference's per-block distortions and
scales bit for bit (mtc/core/allocation.py:106-160); the resulting quadtree
allocations must equal the reference's on the golden inputs.
"""

import os

import numpy as np
import pytest

import inputs

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    import torch

    from tensorpack_b200 import build

    assert torch.cuda.is_available()
    build.build()
    return torch.device("cuda", 0)


def load(golden_dir, name):
    return np.load(os.path.join(golden_dir, name))


def test_candidate_tables_match_reference(golden_dir, dev):
    from tensorpack_b200.quant import QuadtreeRD

    g = load(golden_dir, "qt_outlier_128.npz")
    qt = QuadtreeRD(inputs.outlier_matrix(128, seed=0), None, (32, 16, 8, 4), device=dev)
    for s in (32, 16, 8, 4):
        lv = qt.levels[s]
        np.testing.assert_array_equal(lv.S.cpu().numpy(), g[f"cand_S_{s}"])
        D = lv.D.cpu().numpy()
        np.testing.assert_array_equal(D[1:], g[f"cand_D_{s}"][1:])          # searched modes: exact
        np.testing.assert_allclose(D[0], g[f"cand_D_{s}"][0], rtol=1e-12)  # P0: sum order differs


def assert_same_allocation(a, g, prefix):
    for s in a.sizes:
        np.testing.assert_array_equal(a.leaf[s], g[f"{prefix}leaf_{s}"])
        np.testing.assert_array_equal(a.modes[s], g[f"{prefix}modes_{s}"])
        np.testing.assert_array_equal(a.scales[s], g[f"{prefix}scales_{s}"])
    assert a.total_bits == int(g[prefix + "total_bits"])


@pytest.mark.parametrize("b", [2.0, 3.0, 4.5, 7.0])
def test_quadtree_select_matches_reference(golden_dir, dev, b):
    from tensorpack_b200.quant import QuadtreeRD

    g = load(golden_dir, "qt_outlier_128.npz")
    qt = QuadtreeRD(inputs.outlier_matrix(128, seed=0), None, (32, 16, 8, 4), device=dev)
    assert_same_allocation(qt.select(b), g, f"b{b}_")


@pytest.mark.parametrize("b", [3.125, 4.25])
def test_permuted_llm_like_matches_reference(golden_dir, dev, b):
    from tensorpack_b200.quant import PermutedQuadtreeRD

    g = load(golden_dir, "llm_like_256x512.npz")
    W, h = inputs.llm_like(256, 512, seed=1)
    a = PermutedQuadtreeRD(W, h, (32, 16, 8, 4), device=dev).select(b)
    np.testing.assert_array_equal(a.row_perm, g[f"b{b}_row_perm"])
    np.testing.assert_array_equal(a.col_perm, g[f"b{b}_col_perm"])
    assert_same_allocation(a.inner, g, f"b{b}_inner_")
    assert a.total_bits == int(g[f"b{b}_total_bits"])


def test_cpu_ref_config_matches_reference(golden_dir, dev):
    from tensorpack_b200.quant import QuadtreeRD

    g = load(golden_dir, "cpu_ref_1024.npz")
    W, h, _ = inputs.cpu_ref_config()
    assert_same_allocation(QuadtreeRD(W, h, (32, 16, 8, 4), device=dev).select(3.125), g, "")


def test_allocation_packs_and_dequantises_exactly(golden_dir, dev):
    """GPU-allocated MTC-QT-P matrix -> pack -> GPU dequant == oracle rebuild."""
    from oracle import mtc_oracle as O
    from tensorpack_b200.kernels.gemm import MTCMatrix
    from tensorpack_b200.quant import PermutedQuadtreeRD

    W, h = inputs.llm_like(256, 512, seed=1)
    a = PermutedQuadtreeRD(W, h, (32, 16, 8, 4), device=dev).select(4.25)
    m = MTCMatrix.from_qt_allocation(W, a)
    ref = O.permuted_quadtree_dequant(W, a.row_perm, a.col_perm, a.inner.sizes, a.inner.leaf, a.inner.modes,
                                      a.inner.scales)
    assert np.array_equal(m.to_array(), ref)
    assert m.accounted_bits == a.total_bits
