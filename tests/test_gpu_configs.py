"""The BASELINE configurations as GPU parity cases, at their full sizes.

Each case allocates on the GPU (the allocator itself is checked bit for bit
against the reference on the golden inputs in test_gpu_alloc.py), packs, and
checks:
  * the GPU dequant of the packed matrix equals the oracle rebuild of the same
    allocation bit for bit (mtc/core/quadtree.py:157-171,
    mtc/core/permutation.py:76-79), and the packed bits equal the allocation's
    accounted bits (tests/test_allocation.py:85-86);
  * Y = mtc_gemm(X, W) (the strip-stream decode for M <= 4, the tcgen05
    decode for M <= 16, the prefill kernel above) is within the north-star
    relative Frobenius error 2e-3 (mtc/eval/reference.py:31-38) of the fp64
    product with that dequant, and within 1e-5 of the fp64 product of the
    exact operands the kernel forms (accumulation order only; for the strip
    decode q * fp16(fp16(x) fp16(s 2^e)), tests/strip_emul.py).  The second
    bound grows in
    proportion to K beyond K = 4096: the prefill accumulates the whole
    reduction in one fp32 TMEM accumulator, one rounding per 16-deep MMA
    step, and at K = 14336 (896 steps) its error against the exact product
    measured 1.6e-5.

The fp64 products run on the GPU through torch: they are the checker, not the
path under test.  Inputs are seeded synthetic stand-ins with the shapes and
value distributions the configurations name (Student-t(4) * 0.02 weights with
importance from 1 %-outlier calibration activations; the multi-scale stress
matrix; N(0, 1) for the CPU reference configuration).
"""

import numpy as np
import pytest

import inputs
from oracle import mtc_oracle as O
from test_gpu_parity import TOL_F16, TOL_REF

pytestmark = pytest.mark.gpu

SIZES = (32, 16, 8, 4)


@pytest.fixture(scope="module")
def dev():
    import torch

    from tensorpack_b200 import build

    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    build.build()
    return torch.device("cuda", 0)


def rel_frob(ref, pred):
    """relative_frobenius_error (fp64) on device tensors."""
    import torch

    d = torch.linalg.vector_norm(ref - pred.double())
    n = torch.linalg.vector_norm(ref)
    return float(d / n) if float(n) > 1e-12 else float(d)


def allocate(W, h, bits, permuted, dev):
    """GPU allocation -> packed MTCMatrix and the oracle rebuild in stored order."""
    from tensorpack_b200.kernels.gemm import MTCMatrix
    from tensorpack_b200.quant import PermutedQuadtreeRD, QuadtreeRD

    if permuted:
        a = PermutedQuadtreeRD(W, h, SIZES, device=dev).select(bits)
        inner, pr, pc = a.inner, a.row_perm, a.col_perm
        Ws = W[pr][:, pc]
    else:
        a = QuadtreeRD(W, h, SIZES, device=dev).select(bits)
        inner, pr, pc = a, None, None
        Ws = W
    m = MTCMatrix.from_qt_allocation(W, a)
    assert m.accounted_bits == a.total_bits
    stored = O.quadtree_dequant(Ws, inner.sizes, inner.leaf, inner.modes, inner.scales)
    return m, stored, pr, pc


def check_layer(m, stored, pr, pc, Xs, dev):
    """Bit-exact dequant, then the GEMM for every activation matrix in Xs."""
    import torch

    from tensorpack_b200.kernels.gemm import mtc_gemm

    deq = stored if pr is None else O.unpermute(stored, pr, pc)
    assert np.array_equal(m.to_array(), deq)
    from strip_emul import emulated_product_torch
    from test_gpu_parity import uses_strip

    ds = m.device_stream(dev)
    W64 = torch.from_numpy(deq).to(dev).double()
    w16 = torch.from_numpy(O.fp16_weight_oracle(stored, ds.exp2)).to(dev).double() * 2.0 ** (-ds.exp2)
    del deq
    pr_t = None if pr is None else torch.from_numpy(np.asarray(pr, np.int64)).to(dev)
    pc_t = None if pc is None else torch.from_numpy(np.asarray(pc, np.int64)).to(dev)
    for X in Xs:
        Xt = X if isinstance(X, torch.Tensor) else torch.from_numpy(X).to(dev)
        Y = mtc_gemm(Xt, m)
        torch.cuda.synchronize()
        ds.check_status()
        assert Y.shape == (Xt.shape[0], m.shape[1]) and Y.dtype == torch.float32
        X64 = Xt.double()
        e_ref = rel_frob(X64 @ W64, Y)
        if uses_strip(ds, Xt.shape[0]):  # exact operands of the strip-stream decode
            x16 = Yp = None
            ref16 = emulated_product_torch(m, stored, Xt.float(), ds.strip().host.exp2)
        else:
            x16 = (Xt if pr_t is None else Xt[:, pr_t]).half().double()
            Yp = x16 @ w16
            if pc_t is None:
                ref16 = Yp
            else:
                ref16 = torch.empty_like(Yp)
                ref16[:, pc_t] = Yp
        e16 = rel_frob(ref16, Y)
        print(f"K={m.shape[0]} N={m.shape[1]} M={Xt.shape[0]}: vs reference dequant {e_ref:.3e}, "
              f"vs fp16 operands {e16:.3e}")
        assert e_ref < TOL_REF, (Xt.shape[0], e_ref)
        assert e16 < TOL_F16 * max(1.0, m.shape[0] / 4096), (Xt.shape[0], e16)
        del Y, X64, x16, Yp, ref16
    torch.cuda.empty_cache()


def test_cpu_reference_config(dev):
    """W 1024x1024 ~N(0,1), QuadtreeRD(W, h, (32, 16, 8, 4)).select(3.125), X 256x1024."""
    W, h, X = inputs.cpu_ref_config()
    m, stored, _, _ = allocate(W, h, 3.125, False, dev)
    check_layer(m, stored, None, None, [X, X[:1]], dev)


def test_llm_like_single_layer(dev):
    """W 4096x4096 Student-t(4) * 0.02, MTC-QT-P at 4.25, M in {1, 16, 512}."""
    W, h = inputs.llm_like(4096, 4096, seed=3)
    m, stored, pr, pc = allocate(W, h, 4.25, True, dev)
    Xs = [inputs.llm_activations(M, 4096, seed=10 + M, outlier_seed=3) for M in (1, 16, 512)]
    check_layer(m, stored, pr, pc, Xs, dev)


@pytest.mark.parametrize("K,N", [(896, 896), (896, 128), (896, 4864), (4864, 896)],
                         ids=["q_o", "k_v", "gate_up", "down"])
def test_qwen_stack_shapes(dev, K, N):
    """the four linear shapes of the Qwen2.5-0.5B-shaped stack, MTC-QT-P at 3.125,
    prefill M = 2048 and decode M = 1."""
    W, h = inputs.llm_like(K, N, seed=K + N)
    m, stored, pr, pc = allocate(W, h, 3.125, True, dev)
    Xs = [inputs.llm_activations(M, K, seed=20 + M, outlier_seed=K) for M in (1, 2048)]
    check_layer(m, stored, pr, pc, Xs, dev)


@pytest.mark.parametrize("K,N,Ms", [(4096, 1024, (1, 16, 4096)), (14336, 4096, (1, 16, 4096)),
                                    (4096, 14336, (1, 4096))], ids=["k_v", "down", "gate_up"])
def test_llama_shapes(dev, K, N, Ms):
    """Llama-3-8B-shaped linears at 4.5 b/w, M in {1, 16, 4096} (q/o is the 4096x4096 shape of
    the single-layer case)."""
    W, h = inputs.llm_like(K, N, seed=7)
    m, stored, pr, pc = allocate(W, h, 4.5, True, dev)
    Xs = [inputs.llm_activations(M, K, seed=30 + M, outlier_seed=7) for M in Ms]
    check_layer(m, stored, pr, pc, Xs, dev)


def test_multiscale_stress(dev):
    """W 8192x8192 with per-32x32-block variance log-uniform on [1e-3, 1e2], unpermuted
    QuadtreeRD at 2.5 b/w, X 8192x8192 bf16 ~N(0, 1)."""
    import torch

    W = inputs.multiscale(8192, seed=4)
    m, stored, _, _ = allocate(W, None, 2.5, False, dev)
    g = torch.Generator(device=dev).manual_seed(4)
    X = torch.randn(8192, 8192, generator=g, device=dev).to(torch.bfloat16)
    check_layer(m, stored, None, None, [X, X[:1]], dev)
