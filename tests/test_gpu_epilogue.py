"""Fused output epilogue (bias + activation) and permutation folding on the GPU.

The epilogue is applied by the kernel that writes Y: the decode reduction
(M <= 16), the prefill store loop (unpermuted output) or the column scatter
(permuted output, and the multi-GPU shard assembly).  Its input is the same
fp32 product the plain call writes, so against a torch fp32 reference of the
same op applied to the plain result: the bias add and ReLU are bit-exact, and
SiLU / GELU(tanh) agree to a few ulp (expf / tanhf against torch's
functions; tolerance rtol 1e-5, atol 1e-6).  End to end the layer must match
the oracle's fp64 act(X @ W + b) within the GEMM tolerance, and a folded
chain b'(a'(X)) must equal b(a(X)) bit for bit.
"""

import numpy as np
import pytest

import inputs
from oracle import mtc_oracle as O
from test_gpu_parity import TOL_REF

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    import torch

    from tensorpack_b200 import build

    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    build.build()
    return torch.device("cuda", 0)


def _torch_act(y, act):
    import torch

    if act is None:
        return y
    if act == "relu":
        return torch.relu(y)
    if act == "silu":
        return torch.nn.functional.silu(y)
    return torch.nn.functional.gelu(y, approximate="tanh")


def _matrix(K, N, permuted, seed):
    from tensorpack_b200.kernels.gemm import MTCMatrix

    W, sizes, leaf, modes, scales = inputs.forced_mode_allocation(K, N, seed=seed, p_split=0.5)
    inner = O.QuadtreeAllocation(sizes, leaf, modes, scales, None, 0)
    if not permuted:
        return MTCMatrix.from_qt_allocation(W, inner), O.quadtree_dequant(W, sizes, leaf, modes, scales)
    rng = np.random.default_rng(seed)
    pr, pc = rng.permutation(K), rng.permutation(N)
    m = MTCMatrix.from_qt_allocation(W, O.PermutedAllocation(inner, pr, pc, None, 0))
    return m, O.permuted_quadtree_dequant(W, pr, pc, sizes, leaf, modes, scales)


@pytest.mark.parametrize("permuted", [False, True])
@pytest.mark.parametrize("M", [1, 9, 16, 40, 300])
def test_epilogue_matches_torch_reference(dev, permuted, M):
    import torch

    from tensorpack_b200.kernels.gemm import gemm_fused

    m, _ = _matrix(160, 544, permuted, seed=M + 7 * permuted)
    ds = m.device_stream(dev)
    X = torch.from_numpy(inputs.llm_activations(M, 160, seed=M, outlier_seed=1)).to(dev)
    Y0 = torch.empty(M, 544, device=dev)
    ds.matmul(X, Y0)
    bias = torch.randn(544, device=dev)
    for act in (None, "relu", "silu", "gelu_tanh"):
        for b in (None, bias):
            if b is None and act is None:
                continue
            Y = gemm_fused(X, m, b, act)
            torch.cuda.synchronize()
            ds.check_status()
            ref = _torch_act(Y0 + b if b is not None else Y0, act)
            if act in (None, "relu"):
                assert torch.equal(Y, ref), (act, b is not None)
            else:
                torch.testing.assert_close(Y, ref, rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("M", [3, 200])
def test_layer_with_activation_matches_oracle(dev, M):
    import torch

    from tensorpack_b200.nn.layers import LinearMTCAdaptive

    m, deq = _matrix(192, 800, True, seed=31)
    rng = np.random.default_rng(2)
    b = rng.standard_normal(800).astype(np.float32)
    layer = LinearMTCAdaptive.from_mtc(m, b, activation="silu")
    Xn = inputs.llm_activations(M, 192, seed=3, outlier_seed=1)
    Y = layer(torch.from_numpy(Xn).to(dev)).cpu().numpy()
    z = Xn.astype(np.float64) @ deq.astype(np.float64) + b
    ref = z / (1.0 + np.exp(-z))
    assert O.relative_frobenius_error(ref, Y) < TOL_REF
    # the numpy path of the layer gives the same values within fp32 rounding
    Yn = layer(Xn)
    np.testing.assert_allclose(Yn, Y, rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("act", ["relu", "gelu_tanh"])
@pytest.mark.parametrize("M", [1, 12, 260])
def test_folded_chain_matches_unfolded(dev, M, act):
    """b'(a'(X)) against b(a(X)): a' writes a's values in stored column order
    and b' gathers them back, so with ReLU the chains agree bit for bit; with
    GELU the activation runs in another kernel of the same formula (prefill
    store loop instead of the column scatter), so to a few ulp."""
    import torch

    from tensorpack_b200.nn.layers import LinearMTCAdaptive, fold_layers

    ma, _ = _matrix(128, 384, True, seed=41)
    mb, _ = _matrix(384, 256, True, seed=42)
    rng = np.random.default_rng(4)
    a = LinearMTCAdaptive.from_mtc(ma, rng.standard_normal(384).astype(np.float32), activation=act)
    b = LinearMTCAdaptive.from_mtc(mb, rng.standard_normal(256).astype(np.float32))
    X = torch.from_numpy(inputs.llm_activations(M, 128, seed=M, outlier_seed=2)).to(dev)
    ref_mid = a(X)
    ref = b(ref_mid)
    a2, b2 = fold_layers(a, b)
    assert a2.W_mtc.col_perm is None and a2.W_mtc.arena is ma.arena
    mid = a2(X)
    out = b2(mid)
    torch.cuda.synchronize()
    stored = ref_mid[:, torch.from_numpy(ma.col_perm).to(dev)]
    if act == "relu":
        assert torch.equal(mid, stored)
        assert torch.equal(out, ref)
    else:
        torch.testing.assert_close(mid, stored, rtol=1e-5, atol=1e-6)
        torch.testing.assert_close(out, ref, rtol=1e-4, atol=1e-4)


def test_shard_assembly_epilogue(dev):
    import torch

    from tensorpack_b200 import _lib
    from tensorpack_b200.kernels.device import epilogue

    lib = _lib.load()
    rng = np.random.default_rng(8)
    nseg, seg_len, M = 3, 512, 70
    segs = rng.standard_normal((nseg, M, seg_len)).astype(np.float32)
    N = nseg * seg_len - 5
    pos = rng.permutation(nseg * seg_len)[:N].astype(np.int32)
    src = torch.from_numpy(segs).to(dev)
    p = torch.from_numpy(pos).to(dev)
    bias = torch.randn(N, device=dev)
    Y = torch.empty(M, N, device=dev)
    ep = epilogue(bias, "relu")
    _lib.check(lib.mtc_permute_rows(src.data_ptr(), M * seg_len, seg_len, nseg, seg_len, p.data_ptr(), N, M,
                                    Y.data_ptr(), N, _lib.ctypes.byref(ep),
                                    torch.cuda.current_stream(dev).cuda_stream), "permute_rows")
    torch.cuda.synchronize()
    rows = np.concatenate([segs[g] for g in range(nseg)], axis=1)[:, pos]
    ref = torch.relu(torch.from_numpy(rows).to(dev) + bias)
    assert torch.equal(Y, ref)


def test_bad_activation_code_rejected(dev):
    import torch

    from tensorpack_b200 import _lib

    m, _ = _matrix(64, 256, False, seed=1)
    ds = m.device_stream(dev)
    X = torch.randn(4, 64, device=dev)
    Y = torch.empty(4, 256, device=dev)
    with pytest.raises(ValueError, match="activation"):
        ds.decode(X, Y, _lib.Epilogue(bias=None, act=9))
