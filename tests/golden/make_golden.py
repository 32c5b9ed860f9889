"""Generate the golden fixtures under tests/golden/ from the reference itself.

Run in a container where the Sharexi/TensorPack sources are available (the
path is taken from MTC_REFERENCE_ROOT, default: the read-only mount used when
these fixtures were made).  The GPU box never runs this script: the fixtures
it writes are committed and travel with the repository.

Every input matrix is regenerated from a seed by ``tests/golden/inputs.py``,
so the fixtures hold only the reference's outputs (allocation grids, codes,
arena bytes, checksums), which keeps them small.

    python tests/golden/make_golden.py
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

from mtc.core.allocation import rd_allocate, rd_allocate_pair, rd_candidates  # noqa: E402
from mtc.core.permutation import PermutedQuadtreeRD  # noqa: E402
from mtc.core.quadtree import QuadtreeRD  # noqa: E402
from mtc.kernels.gemm import MTCMatrix, mtc_gemm  # noqa: E402


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def qt_fields(prefix, a, out):
    for s in a.sizes:
        out[f"{prefix}leaf_{s}"] = a.leaf[s]
        out[f"{prefix}modes_{s}"] = a.modes[s]
        out[f"{prefix}scales_{s}"] = a.scales[s]
    out[f"{prefix}sizes"] = np.array(a.sizes)
    out[f"{prefix}total_bits"] = np.array(a.total_bits)
    out[f"{prefix}dequant_sha"] = np.array(sha(a.dequant))


def save(name, **arrays):
    path = os.path.join(HERE, name)
    np.savez_compressed(path, **arrays)
    print("wrote", path, os.path.getsize(path), "bytes")


def main():
    # 1. MTC-QT on a sparse-outlier matrix, sizes 32..4, several budgets.
    W = inputs.outlier_matrix(128, seed=0)
    qt = QuadtreeRD(W, None, (32, 16, 8, 4))
    out = {}
    for b in (2.0, 3.0, 4.5, 7.0):
        a = qt.select(b)
        qt_fields(f"b{b}_", a, out)
        out[f"b{b}_dequant"] = a.dequant
    for s in (32, 16, 8, 4):
        out[f"cand_D_{s}"] = qt.cands[s].D
        out[f"cand_S_{s}"] = qt.cands[s].S
    save("qt_outlier_128.npz", **out)

    # 2. MTC-QT-P on rows of very different scale, sizes (32,16,8) and (32..4).
    W, h = inputs.row_scaled(256, 256, seed=0)
    out = {}
    for sizes, b in (((32, 16, 8), 3.0), ((32, 16, 8, 4), 4.25)):
        a = PermutedQuadtreeRD(W, h, sizes).select(b)
        tag = f"s{len(sizes)}_"
        qt_fields(tag + "inner_", a.inner, out)
        out[tag + "row_perm"] = a.row_perm
        out[tag + "col_perm"] = a.col_perm
        out[tag + "total_bits"] = np.array(a.total_bits)
        out[tag + "dequant"] = a.dequant
    save("qtp_rows_256.npz", **out)

    # 3. LLM-like layer (Student-t weights, outlier input channels), MTC-QT-P.
    W, h = inputs.llm_like(256, 512, seed=1)
    out = {}
    for b in (3.125, 4.25):
        a = PermutedQuadtreeRD(W, h, (32, 16, 8, 4)).select(b)
        tag = f"b{b}_"
        qt_fields(tag + "inner_", a.inner, out)
        out[tag + "row_perm"] = a.row_perm
        out[tag + "col_perm"] = a.col_perm
        out[tag + "total_bits"] = np.array(a.total_bits)
        out[tag + "dequant_sha"] = np.array(sha(a.dequant))
    save("llm_like_256x512.npz", **out)

    # 4. Multi-scale stress stand-in, unpermuted MTC-QT at 2.5 b/w.
    W = inputs.multiscale(256, seed=2)
    a = QuadtreeRD(W, None, (32, 16, 8, 4)).select(2.5)
    out = {}
    qt_fields("", a, out)
    save("multiscale_256.npz", **out)

    # 5. CPU-reference configuration of the benchmark (1024^2, QuadtreeRD @ 3.125).
    W, h, _ = inputs.cpu_ref_config()
    a = QuadtreeRD(W, h, (32, 16, 8, 4)).select(3.125)
    out = {}
    qt_fields("", a, out)
    save("cpu_ref_1024.npz", **out)

    # 6. Fixed 16x16 MTC-RD pair: packed arena, offsets and the packed GEMM.
    A, B = inputs.fixed_pair(seed=5)
    out = {}
    for b in (2.6, 5.2, 9.0):
        aa, bb = rd_allocate_pair(A, B, b)
        Am = MTCMatrix.from_allocation(A, aa.modes, aa.scales, 16)
        Bm = MTCMatrix.from_allocation(B, bb.modes, bb.scales, 16)
        tag = f"b{b}_"
        for nm, al, mm in (("A", aa, Am), ("B", bb, Bm)):
            out[tag + nm + "_modes"] = al.modes
            out[tag + nm + "_scales"] = al.scales
            out[tag + nm + "_dequant"] = al.dequant
            out[tag + nm + "_payload_bits"] = np.array(al.payload_bits)
            out[tag + nm + "_arena"] = mm.arena.raw_buffer[: mm.total_bytes_allocated].copy()
            out[tag + nm + "_offsets"] = mm.offsets
        out[tag + "gemm"] = mtc_gemm(Am, Bm)
    save("fixed_pair.npz", **out)

    # 7. Fixed 16x16 MTC-RD with bf16 scales and importance (the CPU-baseline operand kind).
    W, h = inputs.llm_like(256, 256, seed=3)
    al = rd_allocate(W, 3.125, h, 16, scale_format="bf16")
    c = rd_candidates(W, h, 16, scale_format="bf16")
    save("fixed_bf16_256.npz", modes=al.modes, scales=al.scales, dequant=al.dequant,
         payload_bits=np.array(al.payload_bits), meta_bits=np.array(al.meta_bits),
         cand_D=c.D, cand_S=c.S)

    # 8. Legacy adaptive per-block packing (MTCMatrix.from_numpy) as used by
    #    LinearMTCAdaptive, on the layer's own seeded weights and on a
    #    heavy-tailed matrix that reaches the P8 / P16 escape modes.
    out = {}
    for tag, W in (("layer", inputs.linear_fp32_weight(32, 16, seed=42)),
                   ("heavy", inputs.heavy_tailed(64, 64, seed=9))):
        mm = MTCMatrix.from_numpy(W, block_size=16, epsilon=0.05, use_pointer_hierarchy=False)
        out[tag + "_arena"] = mm.arena.raw_buffer[: mm.total_bytes_allocated].copy()
        out[tag + "_offsets"] = mm.offsets
        out[tag + "_precisions"] = mm.precisions
        out[tag + "_scales"] = mm.scales
        out[tag + "_dequant"] = mm.to_array()
    save("legacy_from_numpy.npz", **out)


if __name__ == "__main__":
    main()
