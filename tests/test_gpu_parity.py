"""GPU parity of the repack, the exact dequantisation and the decode GEMM.

Checked through the C ABI (via tensorpack_b200's ctypes binding) against the
CPU oracle and the golden fixtures produced by the reference:
  * dequantised weights must be bit-exact (np.array_equal) against the
    reference dequant (mtc/core/quadtree.py:157-171, permutation.py:76-79,
    gemm.py:510-538);
  * GEMM outputs must be within relative Frobenius error 2e-3 of the fp64
    product with the reference dequant, and within
    1e-5 of the same product computed from the exact operands the kernel
    forms (which isolates accumulation-order differences): fp16(q s 2^e) and
    fp16(x) for the tcgen05 kernels, q and fp16(fp16(x) fp16(s 2^e)) for the
    strip-stream decode that serves M <= 4.
"""

import os

import numpy as np
import pytest

import inputs
from oracle import mtc_oracle as O
from strip_emul import emulated_product

pytestmark = pytest.mark.gpu

TOL_REF = 2e-3   # north-star tolerance vs the reference fp32 GEMM
TOL_F16 = 1e-5   # vs the fp16-operand product (accumulation order only)


@pytest.fixture(scope="module")
def dev():
    import torch

    from tensorpack_b200 import build

    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    build.build()
    return torch.device("cuda", 0)


def load(golden_dir, name):
    return np.load(os.path.join(golden_dir, name))


def qt_from_golden(g, prefix):
    sizes = tuple(int(s) for s in g[prefix + "sizes"])
    return O.QuadtreeAllocation(sizes, {s: g[f"{prefix}leaf_{s}"] for s in sizes},
                                {s: g[f"{prefix}modes_{s}"] for s in sizes},
                                {s: g[f"{prefix}scales_{s}"] for s in sizes}, None, int(g[prefix + "total_bits"]))


def fp16_product(X, W_stored, exp2, pr=None, pc=None):
    """fp64 product of the exact fp16 operands the kernels feed the tensor cores."""
    Xp = X if pr is None else X[:, pr]
    x16 = Xp.astype(np.float16).astype(np.float64)
    w16 = O.fp16_weight_oracle(W_stored, exp2).astype(np.float64) * 2.0 ** (-exp2)
    Yp = x16 @ w16
    if pc is None:
        return Yp
    Y = np.empty_like(Yp)
    Y[:, pc] = Yp
    return Y


def run_gemm(m, X, dev):
    import torch

    from tensorpack_b200.kernels.gemm import mtc_gemm

    Y = mtc_gemm(torch.from_numpy(X).to(dev), m)
    torch.cuda.synchronize()
    m.device_stream(dev).check_status()
    return Y.cpu().numpy()


def uses_strip(ds, M):
    """Whether DeviceStream.matmul runs the strip-stream decode for M tokens
    (the same rule as matmul)."""
    from tensorpack_b200.kernels.device import STRIP_MAX_M

    return M <= STRIP_MAX_M and ds.decode_kernel == "strip" and ds.strip_fits(M)


def check_gemm(m, W_deq_orig, W_stored, X, dev):
    ds = m.device_stream(dev)
    Y = run_gemm(m, X, dev)
    ref = X.astype(np.float64) @ W_deq_orig.astype(np.float64)
    e_ref = O.relative_frobenius_error(ref, Y)
    if uses_strip(ds, X.shape[0]):
        e16 = O.relative_frobenius_error(emulated_product(m, W_deq_orig, X, ds.strip().host.exp2)[0], Y)
    else:
        e16 = O.relative_frobenius_error(fp16_product(X, W_stored, ds.exp2, m.row_perm, m.col_perm), Y)
    assert e_ref < TOL_REF, e_ref
    assert e16 < TOL_F16, e16
    return Y


# --------------------------------------------------------------------------- dequant


@pytest.mark.parametrize("b", [2.0, 3.0, 4.5, 7.0])
def test_dequant_quadtree_bit_exact(golden_dir, dev, b):
    from tensorpack_b200.kernels.gemm import MTCMatrix

    g = load(golden_dir, "qt_outlier_128.npz")
    m = MTCMatrix.from_qt_allocation(inputs.outlier_matrix(128, seed=0), qt_from_golden(g, f"b{b}_"))
    assert np.array_equal(m.to_array(), g[f"b{b}_dequant"])


@pytest.mark.parametrize("sizes", [(32, 16, 8), (32, 16, 8, 4)])
def test_dequant_permuted_bit_exact(golden_dir, dev, sizes):
    from tensorpack_b200.kernels.gemm import MTCMatrix

    g = load(golden_dir, "qtp_rows_256.npz")
    W, _ = inputs.row_scaled(256, 256, seed=0)
    tag = f"s{len(sizes)}_"
    alloc = O.PermutedAllocation(qt_from_golden(g, tag + "inner_"), g[tag + "row_perm"], g[tag + "col_perm"],
                                 None, int(g[tag + "total_bits"]))
    m = MTCMatrix.from_qt_allocation(W, alloc)
    assert np.array_equal(m.to_array(), g[tag + "dequant"])
    stored = m.device_stream(dev).dequant(original_order=False).cpu().numpy()
    assert np.array_equal(stored, g[tag + "dequant"][alloc.row_perm][:, alloc.col_perm])


@pytest.mark.parametrize("b", [3.125, 4.25])
def test_dequant_llm_like_checksum(golden_dir, dev, b):
    import hashlib

    from tensorpack_b200.kernels.gemm import MTCMatrix

    g = load(golden_dir, "llm_like_256x512.npz")
    W, _ = inputs.llm_like(256, 512, seed=1)
    tag = f"b{b}_"
    alloc = O.PermutedAllocation(qt_from_golden(g, tag + "inner_"), g[tag + "row_perm"], g[tag + "col_perm"],
                                 None, int(g[tag + "total_bits"]))
    d = MTCMatrix.from_qt_allocation(W, alloc).to_array()
    assert hashlib.sha256(np.ascontiguousarray(d).tobytes()).hexdigest() == str(g[tag + "dequant_sha"])


@pytest.mark.parametrize("b", [2.6, 5.2, 9.0])
def test_dequant_fixed_blocks_fp32_scales(golden_dir, dev, b):
    from tensorpack_b200.kernels.gemm import MTCMatrix

    g = load(golden_dir, "fixed_pair.npz")
    A, B = inputs.fixed_pair(seed=5)
    tag = f"b{b}_"
    for nm, X in (("A", A), ("B", B)):
        m = MTCMatrix.from_allocation(X, g[tag + nm + "_modes"], g[tag + nm + "_scales"], 16)
        assert np.array_equal(m.to_array(), g[tag + nm + "_dequant"])


@pytest.mark.parametrize("tag", ["layer", "heavy"])
def test_dequant_legacy_from_numpy(golden_dir, dev, tag):
    from tensorpack_b200.kernels.gemm import MTCMatrix

    g = load(golden_dir, "legacy_from_numpy.npz")
    W = inputs.linear_fp32_weight(32, 16, seed=42) if tag == "layer" else inputs.heavy_tailed(64, 64, seed=9)
    m = MTCMatrix.from_numpy(W, block_size=16, epsilon=0.05, use_pointer_hierarchy=False)
    assert np.array_equal(m.to_array(), g[tag + "_dequant"])


def forced(K=256, N=384, seed=0):
    from tensorpack_b200.kernels.gemm import MTCMatrix

    W, sizes, leaf, modes, scales = inputs.forced_mode_allocation(K, N, seed=seed, p_split=0.5)
    alloc = O.QuadtreeAllocation(sizes, leaf, modes, scales, None, 0)
    deq = O.quadtree_dequant(W, sizes, leaf, modes, scales)
    return MTCMatrix.from_qt_allocation(W, alloc), deq, (sizes, leaf, modes)


def test_forced_modes_cover_every_edge_and_mode(dev):
    m, deq, (sizes, leaf, modes) = forced()
    seen = {(s, int(md)) for s in sizes for md in np.unique(modes[s][leaf[s]])}
    assert seen == {(s, md) for s in sizes for md in (0, 2, 3, 4, 5, 6, 8, 16)}
    assert np.array_equal(m.to_array(), deq)


def test_ragged_shape_dequant_and_gemm(dev):
    from tensorpack_b200.kernels.gemm import MTCMatrix

    rng = np.random.default_rng(3)
    W = rng.standard_normal((48, 80)).astype(np.float32)
    modes = rng.choice([0, 2, 3, 4, 5, 6, 8, 16], size=(3, 5)).astype(np.uint8)
    qmax = np.array([1.0 if x in (0, 2) else 2.0 ** (int(x) - 1) - 1 for x in modes.ravel()]).reshape(3, 5)
    scales = (np.abs(W.reshape(3, 16, 5, 16)).max(axis=(1, 3)) / qmax).astype(np.float32)
    m = MTCMatrix.from_allocation(W, modes, scales, 16)
    deq = O.fixed_dequant(W, modes, np.where(modes == 0, 0, scales).astype(np.float32), 16)
    assert np.array_equal(m.to_array(), deq)
    X = rng.standard_normal((5, 48)).astype(np.float32)
    check_gemm(m, deq, deq, X, dev)


# --------------------------------------------------------------------------- decode GEMM


@pytest.mark.parametrize("M", [1, 2, 7, 8, 9, 16])
def test_gemv_llm_like_permuted(golden_dir, dev, M):
    from tensorpack_b200.kernels.gemm import MTCMatrix

    g = load(golden_dir, "llm_like_256x512.npz")
    W, _ = inputs.llm_like(256, 512, seed=1)
    tag = "b4.25_"
    inner = qt_from_golden(g, tag + "inner_")
    pr, pc = g[tag + "row_perm"], g[tag + "col_perm"]
    alloc = O.PermutedAllocation(inner, pr, pc, None, int(g[tag + "total_bits"]))
    m = MTCMatrix.from_qt_allocation(W, alloc)
    stored = O.quadtree_dequant(W[pr][:, pc], inner.sizes, inner.leaf, inner.modes, inner.scales)
    X = inputs.llm_activations(M, 256, seed=M, outlier_seed=1)
    check_gemm(m, O.unpermute(stored, pr, pc), stored, X, dev)


@pytest.mark.parametrize("M", [1, 16])
def test_gemv_forced_modes(dev, M):
    m, deq, _ = forced()
    X = np.random.default_rng(M).standard_normal((M, 256)).astype(np.float32)
    check_gemm(m, deq, deq, X, dev)


@pytest.mark.parametrize("M", [1, 5, 16])
def test_cuda_core_gemv_matches_reference(golden_dir, dev, M):
    """mtc_gemv (split-K mma.sync kernel, also behind mtc_gemv_static) against the reference and against the
    tensor-core mtc_decode (mtc_gemm routes M <= 4 to the strip decode and 5..16 to mtc_decode)."""
    import torch

    from tensorpack_b200.kernels.gemm import MTCMatrix

    g = load(golden_dir, "llm_like_256x512.npz")
    W, _ = inputs.llm_like(256, 512, seed=1)
    tag = "b4.25_"
    inner = qt_from_golden(g, tag + "inner_")
    pr, pc = g[tag + "row_perm"], g[tag + "col_perm"]
    m = MTCMatrix.from_qt_allocation(W, O.PermutedAllocation(inner, pr, pc, None, int(g[tag + "total_bits"])))
    stored = O.quadtree_dequant(W[pr][:, pc], inner.sizes, inner.leaf, inner.modes, inner.scales)
    X = inputs.llm_activations(M, 256, seed=M + 40, outlier_seed=1)
    ds = m.device_stream(dev)
    Xt = torch.from_numpy(X).to(dev)
    Y1 = torch.empty(M, 512, device=dev)
    Y2 = torch.empty(M, 512, device=dev)
    ds.gemv(Xt, Y1)
    ds.decode(Xt, Y2)
    torch.cuda.synchronize()
    ds.check_status()
    ref = X.astype(np.float64) @ O.unpermute(stored, pr, pc).astype(np.float64)
    assert O.relative_frobenius_error(ref, Y1.cpu().numpy()) < TOL_REF
    # both compute the exact fp16-operand product; only the accumulation order differs
    assert O.relative_frobenius_error(Y1.double().cpu().numpy(), Y2.cpu().numpy()) < TOL_F16


def test_gemv_multiscale(golden_dir, dev):
    from tensorpack_b200.kernels.gemm import MTCMatrix

    g = load(golden_dir, "multiscale_256.npz")
    W = inputs.multiscale(256, seed=2)
    a = qt_from_golden(g, "")
    m = MTCMatrix.from_qt_allocation(W, a)
    deq = O.quadtree_dequant(W, a.sizes, a.leaf, a.modes, a.scales)
    X = np.random.default_rng(0).standard_normal((4, 256)).astype(np.float32)
    check_gemm(m, deq, deq, X, dev)


def test_gemm_reference_signature(golden_dir, dev):
    """mtc_gemm(A, B) with two packed operands, as in tests/test_allocation.py:83."""
    from tensorpack_b200.kernels.gemm import MTCMatrix, mtc_gemm

    g = load(golden_dir, "fixed_pair.npz")
    A, B = inputs.fixed_pair(seed=5)
    tag = "b5.2_"
    Am = MTCMatrix.from_allocation(A, g[tag + "A_modes"], g[tag + "A_scales"], 16)
    Bm = MTCMatrix.from_allocation(B, g[tag + "B_modes"], g[tag + "B_scales"], 16)
    C = mtc_gemm(Am, Bm)
    assert isinstance(C, np.ndarray) and C.shape == (128, 64) and C.dtype == np.float32
    sim = g[tag + "A_dequant"].astype(np.float64) @ g[tag + "B_dequant"]
    assert O.relative_frobenius_error(sim, C) < TOL_REF


def test_numpy_in_numpy_out_and_empty(dev):
    from tensorpack_b200.kernels.gemm import mtc_gemm

    m, deq, _ = forced(64, 96, seed=4)
    Y = mtc_gemm(np.zeros((0, 64), np.float32), m)
    assert Y.shape == (0, 96)
    X = np.random.default_rng(1).standard_normal((3, 64)).astype(np.float32)
    Y = mtc_gemm(X, m)
    assert isinstance(Y, np.ndarray)
    assert O.relative_frobenius_error(X.astype(np.float64) @ deq, Y) < TOL_REF


def test_repeat_calls_are_deterministic(dev):
    import torch

    from tensorpack_b200.kernels.gemm import mtc_gemm

    m, _, _ = forced(128, 256, seed=5)
    X = torch.randn(16, 128, device=dev)
    Y1 = mtc_gemm(X, m).clone()
    Y2 = mtc_gemm(X, m)
    assert torch.equal(Y1, Y2)


def test_out_of_range_activation_is_reported(dev):
    import torch

    from tensorpack_b200.kernels.gemm import mtc_gemm

    m, _, _ = forced(64, 64, seed=6)
    X = torch.ones(2, 64, device=dev)
    X[1, 3] = 1e6
    with pytest.raises(RuntimeError, match="fp16 range"):
        mtc_gemm(X.cpu().numpy(), m)
    # the stream stays usable afterwards
    Y = mtc_gemm(torch.ones(2, 64, device=dev).cpu().numpy(), m)
    assert np.isfinite(Y).all()


def test_linear_layer_drop_in(dev):
    """LinearMTCAdaptive (mtc/nn/layers.py:115-151) forward on the GPU GEMM."""
    from tensorpack_b200.nn.layers import LinearMTCAdaptive

    X = np.random.default_rng(0).standard_normal((8, 32)).astype(np.float32)
    layer = LinearMTCAdaptive(32, 16, block_size=16, seed=42)
    y = layer.forward(X)
    W = inputs.linear_fp32_weight(32, 16, seed=42)
    y32 = X @ W
    assert y.shape == (8, 16)
    assert np.linalg.norm(y32 - y) / np.linalg.norm(y32) < 0.05   # tests/test_nn.py:30-32
    ydq = X.astype(np.float64) @ layer.W_mtc.to_array()
    assert O.relative_frobenius_error(ydq, y) < TOL_REF
    assert layer.weight_bytes == layer.W_mtc.total_bytes_allocated + 16 * 4
