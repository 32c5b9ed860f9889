"""GPU checks of the row kernels around the prefill GEMM, through the C ABI.

mtc_permute_rows: Y[m][j] = row_m[pos[j]], row_m the concatenation of nseg
segments (the column scatter of MTC-QT-P outputs, mtc/core/permutation.py:
15-21, and the assembly of column shards).  Exact copies, so bit-exact
against numpy.  Both the bulk-copy kernel (aligned segments) and the
one-row-per-CTA fallback (unaligned segments) are covered, with row counts
that do not divide the grid.  The X gather (fp16 conversion + row
permutation) is covered through mtc_gemm_prefill with a strided X whose odd
row stride takes the fallback.
"""

import ctypes

import numpy as np
import pytest

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


def permute(dev, segs, pos, M, ldy, seg_stride, ldp, seg_len):
    import torch

    from tensorpack_b200 import _lib

    lib = _lib.load()
    src = torch.from_numpy(segs).to(dev)
    p = torch.from_numpy(pos.astype(np.int32)).to(dev)
    N = len(pos)
    Y = torch.full((M, ldy), -7.0, dtype=torch.float32, device=dev)
    st = torch.cuda.current_stream(dev).cuda_stream
    _lib.check(lib.mtc_permute_rows(src.data_ptr(), seg_stride, ldp, segs.shape[0], seg_len, p.data_ptr(), N, M,
                                    Y.data_ptr(), ldy, None, st), "permute_rows")
    torch.cuda.synchronize()
    return Y.cpu().numpy()


@pytest.mark.parametrize("nseg,seg_len,M,ldp", [(1, 14336, 333, 14336), (3, 512, 1000, 512), (4, 96, 7, 100),
                                                  (2, 98, 50, 101)])
def test_permute_rows_matches_numpy(dev, nseg, seg_len, M, ldp):
    rng = np.random.default_rng(nseg * 1000 + seg_len)
    segs = rng.standard_normal((nseg, M, ldp)).astype(np.float32)
    N = nseg * seg_len - 3
    pos = rng.permutation(nseg * seg_len)[:N]
    ldy = N + 5
    Y = permute(dev, segs, pos, M, ldy, M * ldp, ldp, seg_len)
    rows = np.concatenate([segs[g, :, :seg_len] for g in range(nseg)], axis=1)
    np.testing.assert_array_equal(Y[:, :N], rows[:, pos])
    assert (Y[:, N:] == -7.0).all()


def test_prefill_strided_x_fallback_gather(dev):
    import torch

    from tensorpack_b200.kernels.gemm import MTCMatrix

    import inputs

    W, sizes, leaf, modes, scales = inputs.forced_mode_allocation(128, 256, seed=5, p_split=0.5)
    m = MTCMatrix.from_qt_allocation(W, O.QuadtreeAllocation(sizes, leaf, modes, scales, None, 0))
    deq = O.quadtree_dequant(W, sizes, leaf, modes, scales)
    ds = m.device_stream(dev)
    big = torch.randn(70, 129, device=dev)
    X = big[:, :128]                      # row stride 129 floats: not 16-byte aligned rows
    Y = torch.empty(70, 256, device=dev)
    ds.prefill(X, Y)
    torch.cuda.synchronize()
    ds.check_status()
    ref = X.double().cpu().numpy() @ deq.astype(np.float64)
    assert O.relative_frobenius_error(ref, Y.cpu().numpy()) < TOL_REF
