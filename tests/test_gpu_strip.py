"""GPU parity of the strip-stream decode kernel (mtc_strip_decode, M <= 4).

Through the C ABI (DeviceStream.decode_strip) against:
  * the fp64 product with the reference dequant (mtc/core/quadtree.py:157-171,
    permutation.py:76-79): relative Frobenius error < 2e-3;
  * the exact emulation of the products the kernel forms (tests/strip_emul.py):
    < 1e-5, i.e. fp32 accumulation order only;
and checks the fused epilogue, determinism and the Llama-3-8B gate shape
against the tensor-core decode.
"""

import os

import numpy as np
import pytest

import inputs
from oracle import mtc_oracle as O
from strip_emul import emulated_product

pytestmark = pytest.mark.gpu

TOL_REF = 2e-3
TOL_EMUL = 1e-5


@pytest.fixture(scope="module")
def dev():
    import torch

    from tensorpack_b200 import build

    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    build.build()
    return torch.device("cuda", 0)


def _qt(golden, name, prefix):
    g = np.load(os.path.join(golden, name))
    sizes = tuple(int(s) for s in g[prefix + "sizes"])
    return g, O.QuadtreeAllocation(sizes, {s: g[f"{prefix}leaf_{s}"] for s in sizes},
                                   {s: g[f"{prefix}modes_{s}"] for s in sizes},
                                   {s: g[f"{prefix}scales_{s}"] for s in sizes}, None,
                                   int(g[prefix + "total_bits"]))


def run_strip(m, X, dev, ep=None):
    import torch

    ds = m.device_stream(dev)
    Xd = torch.from_numpy(np.ascontiguousarray(X, dtype=np.float32)).to(dev)
    Y = torch.full((X.shape[0], m.shape[1]), float("nan"), dtype=torch.float32, device=dev)
    ds.decode_strip(Xd, Y, ep)
    torch.cuda.synchronize()
    ds.check_status()
    return Y.cpu().numpy()


def check(m, deq, X, dev):
    Y = run_strip(m, X, dev)
    assert np.isfinite(Y).all()
    e_ref = O.relative_frobenius_error(X.astype(np.float64) @ deq.astype(np.float64), Y)
    emul, _ = emulated_product(m, deq, X, m.device_stream(dev).strip().host.exp2)
    e_emul = O.relative_frobenius_error(emul, Y)
    assert e_ref < TOL_REF, e_ref
    assert e_emul < TOL_EMUL, e_emul
    return Y


def forced(K=256, N=384, seed=0):
    from tensorpack_b200.kernels.gemm import MTCMatrix

    W, sizes, leaf, modes, scales = inputs.forced_mode_allocation(K, N, seed=seed, p_split=0.5)
    alloc = O.QuadtreeAllocation(sizes, leaf, modes, scales, None, 0)
    return MTCMatrix.from_qt_allocation(W, alloc), O.quadtree_dequant(W, sizes, leaf, modes, scales)


@pytest.mark.parametrize("M", [1, 2, 3, 4])
def test_strip_forced_modes(dev, M):
    m, deq = forced()
    X = np.random.default_rng(M).standard_normal((M, 256)).astype(np.float32)
    check(m, deq, X, dev)


@pytest.mark.parametrize("M", [1, 4])
def test_strip_llm_like_permuted(golden_dir, dev, M):
    from tensorpack_b200.kernels.gemm import MTCMatrix

    g, inner = _qt(golden_dir, "llm_like_256x512.npz", "b4.25_inner_")
    W, _ = inputs.llm_like(256, 512, seed=1)
    pr, pc = g["b4.25_row_perm"], g["b4.25_col_perm"]
    m = MTCMatrix.from_qt_allocation(W, O.PermutedAllocation(inner, pr, pc, None, int(g["b4.25_total_bits"])))
    stored = O.quadtree_dequant(W[pr][:, pc], inner.sizes, inner.leaf, inner.modes, inner.scales)
    X = inputs.llm_activations(M, 256, seed=M, outlier_seed=1)
    check(m, O.unpermute(stored, pr, pc), X, dev)


def test_strip_multiscale_and_ragged(golden_dir, dev):
    from tensorpack_b200.kernels.gemm import MTCMatrix

    g, a = _qt(golden_dir, "multiscale_256.npz", "")
    W = inputs.multiscale(256, seed=2)
    m = MTCMatrix.from_qt_allocation(W, a)
    deq = O.quadtree_dequant(W, a.sizes, a.leaf, a.modes, a.scales)
    check(m, deq, np.random.default_rng(0).standard_normal((2, 256)).astype(np.float32), dev)
    rng = np.random.default_rng(3)
    W = rng.standard_normal((48, 80)).astype(np.float32)
    modes = rng.choice([0, 2, 3, 4, 5, 6, 8, 16], size=(3, 5)).astype(np.uint8)
    qmax = np.array([1.0 if x in (0, 2) else 2.0 ** (int(x) - 1) - 1 for x in modes.ravel()]).reshape(3, 5)
    scales = (np.abs(W.reshape(3, 16, 5, 16)).max(axis=(1, 3)) / qmax).astype(np.float32)
    m = MTCMatrix.from_allocation(W, modes, scales, 16)
    deq = O.fixed_dequant(W, modes, np.where(modes == 0, 0, scales).astype(np.float32), 16)
    check(m, deq, rng.standard_normal((3, 48)).astype(np.float32), dev)


def test_strip_epilogue_and_determinism(dev):
    import torch

    from tensorpack_b200.kernels.device import epilogue

    m, deq = forced(seed=3)
    X = np.random.default_rng(9).standard_normal((2, 256)).astype(np.float32)
    Y0 = run_strip(m, X, dev)
    for _ in range(3):  # deterministic: per-batch partials summed in batch order
        assert np.array_equal(run_strip(m, X, dev), Y0)
    bias = torch.from_numpy(np.random.default_rng(1).standard_normal(384).astype(np.float32)).to(dev)
    Y = run_strip(m, X, dev, epilogue(bias, "relu"))
    assert np.array_equal(Y, np.maximum(Y0 + bias.cpu().numpy()[None, :], 0.0))


def test_strip_all_p0_writes_bias(dev):
    import torch

    from tensorpack_b200.kernels.device import epilogue
    from tensorpack_b200.kernels.gemm import MTCMatrix

    m = MTCMatrix.from_allocation(np.zeros((64, 96), np.float32), np.zeros((4, 6), np.uint8),
                                  np.zeros((4, 6), np.float32), 16)
    bias = torch.arange(96, dtype=torch.float32, device=dev)
    Y = run_strip(m, np.ones((1, 64), np.float32), dev, epilogue(bias))
    assert np.array_equal(Y[0], np.arange(96, dtype=np.float32))


def test_strip_gate_shape_matches_tensor_decode(dev):
    """Llama-3-8B gate_proj shape (4096 x 14336, MTC-QT-P at 4.25 b/w,
    allocated on the GPU): the strip kernel and the tensor-core decode agree,
    and the strip stream stays within 1.15x of the accounted bytes."""
    import torch

    from tensorpack_b200.kernels.gemm import MTCMatrix
    from tensorpack_b200.quant import PermutedQuadtreeRD

    W, h = inputs.llm_like(4096, 14336, seed=0)
    alloc = PermutedQuadtreeRD(W, h, (32, 16, 8, 4), device=dev).select(4.25)
    m = MTCMatrix.from_qt_allocation(W, alloc)
    ds = m.device_stream(dev)
    assert ds.strip().stream_bytes < 1.15 * m.accounted_bits / 8
    X = torch.from_numpy(inputs.llm_activations(4, 4096, seed=5, outlier_seed=0)).to(dev)
    for M in (1, 4):
        Ys = torch.empty(M, 14336, dtype=torch.float32, device=dev)
        Yt = torch.empty_like(Ys)
        ds.decode_strip(X[:M], Ys)
        ds.decode(X[:M], Yt)
        torch.cuda.synchronize()
        ds.check_status()
        e = O.relative_frobenius_error(Yt.cpu().numpy().astype(np.float64), Ys.cpu().numpy())
        assert e < 1e-3, (M, e)


def run_form(m, X, dev, wide=False, merge_modes=False, batch_bytes=None):
    """The decode through a non-default strip form of the same matrix."""
    import ctypes

    import torch

    from tensorpack_b200 import _lib

    ds = m.device_stream(dev)
    sp = ds.strip(wide=wide, merge_modes=merge_modes, batch_bytes=batch_bytes)
    Xd = torch.from_numpy(np.ascontiguousarray(X, dtype=np.float32)).to(dev)
    Y = torch.full((X.shape[0], m.shape[1]), float("nan"), dtype=torch.float32, device=dev)
    lib = _lib.load()
    _lib.check(lib.mtc_strip_decode(ctypes.byref(sp.desc_for(X.shape[0])), Xd.data_ptr(), X.shape[0], Xd.stride(0),
                                    None if ds.row_perm is None else ds.row_perm.data_ptr(),
                                    None if ds.col_perm is None else ds.col_perm.data_ptr(), Y.data_ptr(),
                                    Y.stride(0), ds.status.data_ptr(), None,
                                    torch.cuda.current_stream(dev).cuda_stream), "strip decode")
    torch.cuda.synchronize()
    ds.check_status()
    return Y.cpu().numpy(), sp.host.exp2


@pytest.mark.parametrize("form", ["wide", "merge", "wide+merge", "small-batches"])
@pytest.mark.parametrize("M", [1, 2, 4])
def test_strip_forms_match_emulation(dev, form, M):
    """The wide group steps, the merged decoder classes and 2 KB batch
    records give the same products as the default form: within 1e-5 of the
    exact emulation and 2e-3 of the reference dequant, on the forced
    all-modes fixture (every mode at every leaf edge) and the permuted
    LLM-like layer."""
    from tensorpack_b200.kernels.gemm import MTCMatrix

    kw = {"wide": {"wide": True}, "merge": {"merge_modes": True}, "wide+merge": {"wide": True, "merge_modes": True},
          "small-batches": {"batch_bytes": 2048}}[form]
    m, deq = forced()
    X = np.random.default_rng(M + 30).standard_normal((M, 256)).astype(np.float32)
    for mat, d, x in [(m, deq, X)]:
        Y, e2 = run_form(mat, x, dev, **kw)
        emul, _ = emulated_product(mat, d, x, e2)
        assert O.relative_frobenius_error(emul, Y) < TOL_EMUL
        assert O.relative_frobenius_error(x.astype(np.float64) @ d.astype(np.float64), Y) < TOL_REF
    g, inner = _qt(os.path.join(os.path.dirname(__file__), "golden"), "llm_like_256x512.npz", "b4.25_inner_")
    W, _ = inputs.llm_like(256, 512, seed=1)
    pr, pc = g["b4.25_row_perm"], g["b4.25_col_perm"]
    m = MTCMatrix.from_qt_allocation(W, O.PermutedAllocation(inner, pr, pc, None, int(g["b4.25_total_bits"])))
    stored = O.quadtree_dequant(W[pr][:, pc], inner.sizes, inner.leaf, inner.modes, inner.scales)
    deq = O.unpermute(stored, pr, pc)
    X = inputs.llm_activations(M, 256, seed=M + 3, outlier_seed=1)
    Y, e2 = run_form(m, X, dev, **kw)
    emul, _ = emulated_product(m, deq, X, e2)
    assert O.relative_frobenius_error(emul, Y) < TOL_EMUL
    assert O.relative_frobenius_error(X.astype(np.float64) @ deq.astype(np.float64), Y) < TOL_REF
