"""Writes tests/golden/pack_v1.mtcpk: a small MTC-QT-P matrix in container
version 1 of the on-disk format (tensorpack_b200.core.fileformat).

The file pins the format: tests load it with the current reader and check
the matrix (every mode, all four leaf edges, fp32 scales, both permutations)
against the oracle, and check that saving it again gives the same bytes.
Run from the repository root: ``python tests/golden/make_pack_fixture.py``.
"""

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
sys.path.insert(0, HERE)

import inputs  # noqa: E402
from oracle import mtc_oracle as O  # noqa: E402
from tensorpack_b200.kernels.gemm import MTCMatrix  # noqa: E402


def fixture_matrix():
    """The matrix stored in the fixture, rebuilt from seeds."""
    W, sizes, leaf, modes, scales = inputs.forced_mode_allocation(64, 96, seed=21, p_split=0.5)
    # one scale that is not bf16-exact, so the fp32 scale array is exercised
    s4 = scales[4].copy()
    ii, jj = np.nonzero(leaf[4] & (modes[4] != 0))
    s4[ii[0], jj[0]] = np.float32(s4[ii[0], jj[0]]) * np.float32(1.0 + 2.0 ** -20)
    scales = dict(scales)
    scales[4] = s4
    rng = np.random.default_rng(7)
    pr, pc = rng.permutation(64), rng.permutation(96)
    inner = O.QuadtreeAllocation(sizes, leaf, modes, scales, None, 0)
    alloc = O.PermutedAllocation(inner, pr, pc, None, 0)
    return W, alloc, MTCMatrix.from_qt_allocation(W, alloc)


if __name__ == "__main__":
    _, _, m = fixture_matrix()
    m.save(os.path.join(HERE, "pack_v1.mtcpk"))
    print("wrote", os.path.join(HERE, "pack_v1.mtcpk"), os.path.getsize(os.path.join(HERE, "pack_v1.mtcpk")), "bytes")
