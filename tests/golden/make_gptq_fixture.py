"""Generate tests/golden/gptq_qtp_256.npz from the reference itself.

GPTQ codes on an MTC-QT-P grid (the reference's qt_quantizer with GPTQ,
mtc/benchmarks/benchmark_gptq.py:140-161): the reference's
PermutedQuadtreeRD allocates the grid, qt_element_grid expands it to
per-element (scale, lo, hi) in the original order, and gptq(..., "fixed",
act_order=True) chooses the integer codes with second-order error
compensation, so the codes differ from rint(W / s).  Stored: the allocation
(inner grids, permutations), the codes in stored (permuted) order as int16,
and the SHA-256 of the reference's dequantised result Q = codes * s
(original order, fp32, signed zeros as +0.0), which the packed matrix must
reproduce bit for bit.

Run where the Sharexi/TensorPack sources are importable (MTC_REFERENCE_ROOT,
default: the read-only mount used when the fixture was made); the GPU box
only reads the committed fixture.

    python tests/golden/make_gptq_fixture.py
"""

import hashlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
import inputs  # noqa: E402

REF = os.environ.get("MTC_REFERENCE_ROOT", "/root/reference")
sys.path.insert(0, REF)

import torch  # noqa: E402

from mtc.baselines.gptq import gptq, qt_element_grid  # noqa: E402
from mtc.core.permutation import PermutedQuadtreeRD  # noqa: E402


def main():
    W, X = inputs.gptq_layer(256, 256, seed=0)
    H = torch.from_numpy((X.T.astype(np.float64) @ X).astype(np.float32))
    h = torch.diag(H).double().numpy()
    a = PermutedQuadtreeRD(W, h, (32, 16, 8, 4)).select(4.25)
    inner, pr, pc = a.inner, a.row_perm, a.col_perm
    Sp, LOp, HIp = qt_element_grid(inner.sizes, inner.leaf, inner.modes, inner.scales, W.shape)
    S, LO, HI = (np.empty_like(Sp) for _ in range(3))
    ix = np.ix_(pr, pc)
    S[ix], LO[ix], HI[ix] = Sp, LOp, HIp
    t = torch.from_numpy
    Q = gptq(t(W), H, "fixed", t(S), t(LO), t(HI), act_order=True).numpy()
    codes = np.where(S != 0, Q / np.where(S != 0, S, 1), 0)
    assert np.array_equal(codes, np.rint(codes)) and np.abs(codes).max() < 2 ** 15
    codes = codes.astype(np.int16)
    assert np.array_equal(codes.astype(np.float32) * S, Q)
    rtn = np.clip(np.round(W / np.where(S != 0, S, 1)), LO, HI).astype(np.int16)
    out = {"row_perm": pr, "col_perm": pc, "total_bits": np.array(a.total_bits),
           "sizes": np.array(inner.sizes), "codes_stored": codes[pr][:, pc],
           # +0.0 turns GPTQ's -0.0 products into +0.0, the reconstruction
           # convention of qt_dequant (which sums its levels)
           "Q_sha": np.array(hashlib.sha256(np.ascontiguousarray(Q + np.float32(0.0)).tobytes()).hexdigest()),
           "codes_differ_from_rtn": np.array(int((codes != rtn).sum()))}
    for s in inner.sizes:
        out[f"leaf_{s}"], out[f"modes_{s}"], out[f"scales_{s}"] = inner.leaf[s], inner.modes[s], inner.scales[s]
    path = os.path.join(HERE, "gptq_qtp_256.npz")
    np.savez_compressed(path, **out)
    print("wrote", path, os.path.getsize(path), "bytes;", int(out["codes_differ_from_rtn"]), "codes differ from RTN")


if __name__ == "__main__":
    main()
