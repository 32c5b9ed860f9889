"""GPTQ codes (explicit, non-RTN) on an MTC-QT-P grid through the GPU path.

The fixture (tests/golden/make_gptq_fixture.py) holds a reference-made
MTC-QT-P allocation, the integer codes the reference's GPTQ chose on that
grid (mtc/baselines/gptq.py:39-138, qt_element_grid; about a fifth differ
from rint(W / s)) and the SHA-256 of the reference's dequantised result Q.
Packed with MTCMatrix.from_qt_allocation(W, alloc, codes=...), the GPU
dequant must reproduce Q bit for bit and every GEMM kernel must stay within
2e-3 of the fp64 product X @ Q.
"""

import hashlib

import numpy as np
import pytest

from oracle import mtc_oracle as O
from test_host_layout import gptq_fixture

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def gptq_matrix(golden_dir):
    import torch

    from tensorpack_b200 import build
    from tensorpack_b200.kernels.gemm import MTCMatrix

    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    build.build()
    g, a, W, X = gptq_fixture(golden_dir)
    return g, MTCMatrix.from_qt_allocation(W, a, codes=g["codes_stored"]), X


def test_gptq_dequant_bit_exact(gptq_matrix):
    g, m, _ = gptq_matrix
    Q = m.to_array()
    assert hashlib.sha256(np.ascontiguousarray(Q).tobytes()).hexdigest() == str(g["Q_sha"])


@pytest.mark.parametrize("M", [1, 4, 16, 300])
def test_gptq_gemm_against_q(gptq_matrix, M):
    """M = 1, 4: strip decode; 16: tensor-core decode; 300: fused prefill."""
    import torch

    from tensorpack_b200.kernels.gemm import mtc_gemm

    g, m, Xc = gptq_matrix
    Q = m.to_array().astype(np.float64)
    X = np.ascontiguousarray(Xc[:M])
    Y = mtc_gemm(torch.from_numpy(X).cuda(), m).cpu().numpy()
    assert O.relative_frobenius_error(X.astype(np.float64) @ Q, Y) < 2e-3
