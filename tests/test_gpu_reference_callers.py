"""The reference's own hot-path test bodies, run through install_mtc_alias().

``tensorpack_b200.install_mtc_alias()`` makes ``import mtc.kernels.gemm``,
``mtc.nn.layers``, ``mtc.core.quadtree`` and ``mtc.core.permutation``
resolve to this package; the tests below import through those names exactly
as the reference's tests do and keep their assertions and bars:

* tests/test_allocation.py:69-86  bit-exact to_array, mtc_gemm(Am, Bm)
  within 1e-5 of the product of the dequantised operands, arena bytes equal
  to the accounted payload bits (fixed-block allocations written by the
  reference's rd_allocate_pair, tests/golden/fixed_pair.npz);
* tests/test_nn.py:12-32          LinearMTCAdaptive within 5 % of LinearFP32;
* tests/test_quadtree.py:37-40    exact rebuild of an MTC-QT allocation;
* tests/test_permutation.py:30-50 budget with index bits, exact rebuild,
  gather / GEMM / scatter inference on the stored matrix,
plus, for each, the same product through this package's GPU GEMM.
The inputs are this repository's seeded generators (tests/golden/inputs.py),
not the reference's RandomState draws.
"""

import os
import sys

import numpy as np
import pytest

import inputs

pytestmark = pytest.mark.gpu


def _rel(ref, pred):
    return float(np.linalg.norm(ref - pred) / np.linalg.norm(ref))


@pytest.fixture(scope="module", autouse=True)
def alias():
    import torch

    import tensorpack_b200
    from tensorpack_b200 import build

    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    build.build()
    saved = {k: v for k, v in sys.modules.items() if k == "mtc" or k.startswith("mtc.")}
    tensorpack_b200.install_mtc_alias()
    yield
    for k in [k for k in sys.modules if k == "mtc" or k.startswith("mtc.")]:
        del sys.modules[k]
    sys.modules.update(saved)


def test_alias_resolves_to_this_package():
    import mtc.core.permutation as P
    import mtc.kernels.gemm as G
    import mtc.nn.layers as L

    assert G.mtc_gemm.__module__.startswith("tensorpack_b200")
    assert G.MTCMatrix.__module__.startswith("tensorpack_b200")
    assert L.LinearMTCAdaptive.__module__.startswith("tensorpack_b200")
    assert P.PermutedQuadtreeRD.__module__.startswith("tensorpack_b200")


@pytest.mark.parametrize("budget", [2.6, 5.2, 9.0])
def test_packed_kernel_matches_simulation(golden_dir, budget):
    from mtc.kernels.gemm import MTCMatrix, mtc_gemm

    g = np.load(os.path.join(golden_dir, "fixed_pair.npz"))
    A, B = inputs.fixed_pair(seed=5)

    class Alloc:  # the fields of the reference's rd_allocate_pair result that the test reads
        def __init__(self, tag):
            self.modes, self.scales = g[tag + "modes"], g[tag + "scales"]
            self.dequant, self.payload_bits = g[tag + "dequant"], int(g[tag + "payload_bits"])

    a, b = Alloc(f"b{budget}_A_"), Alloc(f"b{budget}_B_")
    Am = MTCMatrix.from_allocation(A, a.modes, a.scales, 16)
    Bm = MTCMatrix.from_allocation(B, b.modes, b.scales, 16)
    np.testing.assert_allclose(Am.to_array(), a.dequant, rtol=0, atol=0)
    np.testing.assert_allclose(Bm.to_array(), b.dequant, rtol=0, atol=0)
    C_sim = a.dequant @ b.dequant
    assert _rel(C_sim, mtc_gemm(Am, Bm)) < 1e-5
    assert Am.total_bytes_allocated * 8 == a.payload_bits
    assert Bm.total_bytes_allocated * 8 == b.payload_bits
    # the hot-path form: activations times the packed right operand
    assert _rel(C_sim, mtc_gemm(np.ascontiguousarray(a.dequant), Bm)) < 2e-3


def test_linear_layers_forward():
    from mtc.nn.layers import LinearFP32, LinearMTCAdaptive

    X = np.random.default_rng(0).standard_normal((8, 32)).astype(np.float32)
    l_fp32 = LinearFP32(32, 16, seed=42)
    l_mtc = LinearMTCAdaptive(32, 16, block_size=16, seed=42)
    y_fp32 = l_fp32.forward(X)
    y_mtc = l_mtc.forward(X)
    assert y_fp32.shape == (8, 16)
    assert y_mtc.shape == (8, 16)
    rel_err_mtc = np.linalg.norm(y_fp32 - y_mtc) / np.linalg.norm(y_fp32)
    assert rel_err_mtc < 0.05


def test_rebuild_is_exact():
    from mtc.core.quadtree import qt_allocate, qt_dequant

    W = inputs.outlier_matrix(128, seed=1)
    a = qt_allocate(W, 3.5)
    np.testing.assert_array_equal(qt_dequant(W, a.sizes, a.leaf, a.modes, a.scales), a.dequant)


@pytest.mark.parametrize("budget", [2.5, 4.25])
def test_budget_includes_index_bits(budget):
    from mtc.core.permutation import PermutedQuadtreeRD, index_bits

    W, h = inputs.row_scaled()
    a = PermutedQuadtreeRD(W, h, (32, 16, 8)).select(budget)
    assert a.bits_per_element <= budget + 1e-9
    assert a.total_bits == a.inner.total_bits + index_bits(*W.shape, True, True)


def test_rebuild_and_gather_scatter_inference_exact():
    from mtc.core.permutation import PermutedQuadtreeRD, permuted_qt_dequant
    from mtc.kernels.gemm import MTCMatrix, mtc_gemm

    W, h = inputs.row_scaled()
    a = PermutedQuadtreeRD(W, h, (32, 16, 8)).select(3.0)
    inner = a.inner
    rebuilt = permuted_qt_dequant(W, a.row_perm, a.col_perm, inner.sizes, inner.leaf, inner.modes, inner.scales)
    np.testing.assert_array_equal(rebuilt, a.dequant)

    X = np.random.default_rng(1).standard_normal((8, W.shape[0])).astype(np.float32)
    Y = np.empty((8, W.shape[1]), np.float32)
    Y[:, a.col_perm] = X[:, a.row_perm] @ inner.dequant
    ref = X @ a.dequant
    assert np.abs(Y - ref).max() <= 1e-6 * np.abs(ref).max()
    # the same inference through the packed GPU GEMM (gather and scatter fused)
    Yg = mtc_gemm(X, MTCMatrix.from_qt_allocation(W, a))
    assert _rel(X.astype(np.float64) @ a.dequant, Yg) < 2e-3
