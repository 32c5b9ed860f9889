"""GPU parity of the fused dequant + tcgen05 prefill GEMM (M > 16 path).

Same bars as the decode tests: relative Frobenius error < 2e-3 against the
fp64 product with the reference dequant, and < 1e-5 against the fp64
product of the exact fp16 operands (isolating accumulation order).
Shapes cover M tails inside a 256-row tile, an odd number of 32-row k tiles
(half-empty last K stage), column bands narrower than 256 and padded
(non-multiple-of-32) matrices.
"""

import os

import numpy as np
import pytest

import inputs
from oracle import mtc_oracle as O
from test_gpu_parity import TOL_F16, TOL_REF, fp16_product, qt_from_golden

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    import torch

    from tensorpack_b200 import build

    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    build.build()
    return torch.device("cuda", 0)


def prefill(m, X, dev):
    import torch

    ds = m.device_stream(dev)
    Xt = torch.from_numpy(X).to(dev)
    Y = torch.empty(X.shape[0], m.shape[1], dtype=torch.float32, device=dev)
    ds.prefill(Xt, Y)
    torch.cuda.synchronize()
    ds.check_status()
    return Y.cpu().numpy()


def check(m, deq_orig, stored, X, dev):
    Y = prefill(m, X, dev)
    ds = m.device_stream(dev)
    e_ref = O.relative_frobenius_error(X.astype(np.float64) @ deq_orig.astype(np.float64), Y)
    e16 = O.relative_frobenius_error(fp16_product(X, stored, ds.exp2, m.row_perm, m.col_perm), Y)
    assert e_ref < TOL_REF, e_ref
    assert e16 < TOL_F16, e16


def llm_matrix(golden_dir):
    from tensorpack_b200.kernels.gemm import MTCMatrix

    g = np.load(os.path.join(golden_dir, "llm_like_256x512.npz"))
    W, _ = inputs.llm_like(256, 512, seed=1)
    inner = qt_from_golden(g, "b4.25_inner_")
    pr, pc = g["b4.25_row_perm"], g["b4.25_col_perm"]
    m = MTCMatrix.from_qt_allocation(W, O.PermutedAllocation(inner, pr, pc, None, 0))
    stored = O.quadtree_dequant(W[pr][:, pc], inner.sizes, inner.leaf, inner.modes, inner.scales)
    return m, O.unpermute(stored, pr, pc), stored


@pytest.mark.parametrize("M", [1, 16, 17, 100, 256, 257, 600])
def test_prefill_llm_like_permuted(golden_dir, dev, M):
    m, deq, stored = llm_matrix(golden_dir)
    X = inputs.llm_activations(M, 256, seed=100 + M, outlier_seed=1)
    check(m, deq, stored, X, dev)


def forced(K, N, seed):
    from tensorpack_b200.kernels.gemm import MTCMatrix

    W, sizes, leaf, modes, scales = inputs.forced_mode_allocation(K, N, seed=seed, p_split=0.5)
    m = MTCMatrix.from_qt_allocation(W, O.QuadtreeAllocation(sizes, leaf, modes, scales, None, 0))
    return m, O.quadtree_dequant(W, sizes, leaf, modes, scales)


@pytest.mark.parametrize("K,N,M", [(256, 384, 40), (256, 384, 300), (96, 160, 70), (32, 32, 33)])
def test_prefill_forced_modes(dev, K, N, M):
    m, deq = forced(K, N, seed=K + N)
    X = np.random.default_rng(M).standard_normal((M, K)).astype(np.float32)
    check(m, deq, deq, X, dev)


def test_prefill_padded_fixed_blocks(dev):
    from tensorpack_b200.kernels.gemm import MTCMatrix

    rng = np.random.default_rng(11)
    W = rng.standard_normal((48, 80)).astype(np.float32)
    modes = rng.choice([0, 2, 3, 4, 5, 6, 8, 16], size=(3, 5)).astype(np.uint8)
    qmax = np.array([1.0 if x in (0, 2) else 2.0 ** (int(x) - 1) - 1 for x in modes.ravel()]).reshape(3, 5)
    scales = (np.abs(W.reshape(3, 16, 5, 16)).max(axis=(1, 3)) / qmax).astype(np.float32)
    m = MTCMatrix.from_allocation(W, modes, scales, 16)
    deq = O.fixed_dequant(W, modes, np.where(modes == 0, 0, scales).astype(np.float32), 16)
    X = rng.standard_normal((45, 48)).astype(np.float32)
    check(m, deq, deq, X, dev)


def test_prefill_matches_decode_kernel(golden_dir, dev):
    """Both kernels compute the same fp16-operand product (M = 16 through each)."""
    import torch

    m, _, _ = llm_matrix(golden_dir)
    ds = m.device_stream(dev)
    X = torch.from_numpy(inputs.llm_activations(16, 256, seed=5, outlier_seed=1)).to(dev)
    Y1 = torch.empty(16, 512, device=dev)
    Y2 = torch.empty(16, 512, device=dev)
    ds.gemv(X, Y1)
    ds.prefill(X, Y2)
    torch.cuda.synchronize()
    ds.check_status()
    err = ((Y1.double() - Y2.double()).norm() / Y2.double().norm()).item()
    assert err < 1e-6, err


def test_mtc_gemm_dispatch_large_m(dev):
    import torch

    from tensorpack_b200.kernels.gemm import mtc_gemm

    m, deq = forced(128, 256, seed=3)
    X = torch.randn(512, 128, device=dev)
    Y = mtc_gemm(X, m)
    ref = X.double().cpu().numpy() @ deq.astype(np.float64)
    assert O.relative_frobenius_error(ref, Y.cpu().numpy()) < TOL_REF


@pytest.mark.parametrize("K,N,M,permuted", [(256, 4096, 3000, False), (160, 4096, 2600, True), (64, 8192, 4400, False)])
def test_prefill_many_tiles(dev, K, N, M, permuted):
    """More pair tiles than CTA pairs (96, 96 and 288 tiles): persistent
    pairs take several tiles each, with the fused epilogue too; the result
    within the GEMM tolerance of the oracle, and the epilogue applied to the
    same sums as the plain call."""
    import torch

    from tensorpack_b200.kernels.device import epilogue
    from tensorpack_b200.kernels.gemm import MTCMatrix

    W, sizes, leaf, modes, scales = inputs.forced_mode_allocation(K, N, seed=K + M, p_split=0.3)
    inner = O.QuadtreeAllocation(sizes, leaf, modes, scales, None, 0)
    if permuted:
        rng = np.random.default_rng(K)
        pr, pc = rng.permutation(K), rng.permutation(N)
        m = MTCMatrix.from_qt_allocation(W, O.PermutedAllocation(inner, pr, pc, None, 0))
        deq = O.permuted_quadtree_dequant(W, pr, pc, sizes, leaf, modes, scales)
    else:
        m = MTCMatrix.from_qt_allocation(W, inner)
        deq = O.quadtree_dequant(W, sizes, leaf, modes, scales)
    X = np.random.default_rng(M).standard_normal((M, K)).astype(np.float32)
    ref = X.astype(np.float64) @ deq.astype(np.float64)
    Y = prefill(m, X, dev)
    assert O.relative_frobenius_error(ref, Y) < TOL_REF
    ds = m.device_stream(dev)
    b = torch.randn(N, device=dev)
    Xt = torch.from_numpy(X).to(dev)
    Ye = torch.empty(M, N, device=dev)
    ds.prefill(Xt, Ye, epilogue(b, "relu"))
    torch.cuda.synchronize()
    ds.check_status()
    refe = np.maximum(ref + b.double().cpu().numpy(), 0.0)
    assert O.relative_frobenius_error(refe, Ye.cpu().numpy()) < TOL_REF
    assert torch.equal(Ye, torch.relu(torch.from_numpy(Y).to(dev) + b))


@pytest.mark.parametrize("M,chunk", [(3000, 1024), (1030, 1024), (10, 1024), (700, 256)])
def test_host_gemm_pipeline(dev, M, chunk):
    """HostGemm: pinned host X in, host Y out, row chunks overlapped.  Rows
    are independent in the GEMM, so chunks of the prefill kernel give the
    whole-matrix call's values up to the summation order: both sum the same
    fp16 operands, but a tail of tiles cut along K is cut by the tile count
    of the call (TOL_F16); a chunk of <= 16 rows goes to the decode kernel
    (another summation order), held to the tolerance."""
    import torch

    from tensorpack_b200.kernels.gemm import HostGemm

    m, deq = forced(256, 640, seed=9)
    X = np.random.default_rng(M).standard_normal((M, 256)).astype(np.float32)
    hg = HostGemm(m, dev, chunk_rows=chunk)
    Xh = torch.from_numpy(X).pin_memory()
    Yh = hg(Xh)
    Yh2 = hg(Xh, torch.empty(M, 640).pin_memory())  # buffers reused
    assert torch.equal(Yh, Yh2)
    ref = X.astype(np.float64) @ deq.astype(np.float64)
    assert O.relative_frobenius_error(ref, Yh.numpy()) < TOL_REF
    whole = prefill(m, X, dev) if M > 16 else None
    if whole is not None and (M % chunk == 0 or M % chunk > 16):
        assert O.relative_frobenius_error(whole.astype(np.float64), Yh.numpy()) < TOL_F16
    with pytest.raises(ValueError):
        hg(torch.zeros(4, 255))
