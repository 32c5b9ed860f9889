"""The decode GEMM entry point that allocates nothing (mtc_gemv_static).

It is for callers that cannot allocate device memory when they run a decode
step (allocator hooks, real-time loops that must not take the allocator's
lock, plugins that only receive inputs and outputs): its split-K scratch is an array built into the library.  Called
through the C ABI, twice in a row, it must agree with the workspace-taking
entry point mtc_gemv within the fp16-operand tolerance of the other GPU tests
(the two may split K differently, so summation order can differ).  The file
name keeps it last in collection order; it also passes alone in a fresh
process because every call clears the shared tickets first.
"""

import ctypes
import os

import numpy as np
import pytest

import inputs

pytestmark = pytest.mark.gpu

TOL = 1e-5  # same bar as the accumulation-order checks of test_gpu_parity.py


def _matrix(golden_dir):
    from oracle import mtc_oracle as O
    from tensorpack_b200.kernels.gemm import MTCMatrix

    g = np.load(os.path.join(golden_dir, "llm_like_256x512.npz"))
    W, _ = inputs.llm_like(256, 512, seed=1)
    sizes = tuple(int(s) for s in g["b4.25_inner_sizes"])
    inner = O.QuadtreeAllocation(sizes, {s: g[f"b4.25_inner_leaf_{s}"] for s in sizes},
                                 {s: g[f"b4.25_inner_modes_{s}"] for s in sizes},
                                 {s: g[f"b4.25_inner_scales_{s}"] for s in sizes}, None, 0)
    return MTCMatrix.from_qt_allocation(W, O.PermutedAllocation(inner, g["b4.25_row_perm"], g["b4.25_col_perm"],
                                                                None, 0))


@pytest.mark.parametrize("M", [1, 16])
def test_static_scratch_decode_matches_workspace_decode(golden_dir, M):
    import torch

    from tensorpack_b200 import _lib, build

    assert torch.cuda.is_available()
    build.build()
    lib = _lib.load()
    dev = torch.device("cuda", 0)
    ds = _matrix(golden_dir).device_stream(dev)
    X = torch.from_numpy(inputs.llm_activations(M, 256, seed=40 + M, outlier_seed=1)).to(dev)
    Y_ref = torch.empty(M, 512, device=dev)
    ds.gemv(X, Y_ref)
    st = torch.cuda.current_stream(dev).cuda_stream
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    pr = ds.row_perm.data_ptr()
    pc = ds.col_perm.data_ptr()
    for call in range(2):
        Y = torch.full((M, 512), float("nan"), device=dev)
        rc = lib.mtc_gemv_static(ctypes.byref(ds.desc), X.data_ptr(), M, X.stride(0), pr, pc, Y.data_ptr(),
                                 Y.stride(0), status.data_ptr(), st)
        assert rc == 0, lib.mtc_last_error()
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        err = ((Y.double() - Y_ref.double()).norm() / Y_ref.double().norm()).item()
        assert err < TOL, (call, err)


def test_static_scratch_decode_rejects_large_m(golden_dir):
    import torch

    from tensorpack_b200 import _lib

    lib = _lib.load()
    dev = torch.device("cuda", 0)
    ds = _matrix(golden_dir).device_stream(dev)
    X = torch.zeros(17, 256, device=dev)
    Y = torch.zeros(17, 512, device=dev)
    rc = lib.mtc_gemv_static(ctypes.byref(ds.desc), X.data_ptr(), 17, 256, None, None, Y.data_ptr(), 512, None,
                             torch.cuda.current_stream(dev).cuda_stream)
    assert rc == _lib.MTC_ERR_INVALID
    assert b"outside 1..16" in lib.mtc_last_error()
