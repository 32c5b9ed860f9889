"""The strip stream (decode-sized device layout) on the CPU.

The stream is built by the native host builder (mtc_strip_plan / _fill) and
consumed by a CPU model of the strip kernel (tests/native/strip_model.cu),
which runs the kernel's own per-lane decode from mtc_strip.cuh for all 32
lanes of every step and evaluates its mma.sync.m16n8k16 fragments with the
PTX layout of that shape.  Checked here:
  * every precision's code placement packs and decodes 16 codes losslessly
    and uses exactly 16 m bits;
  * structural invariants of the batch records;
  * the model's product equals the fp64 product with the reference dequant
    (mtc/core/quadtree.py:157-171, permutation.py:76-79, gemm.py:510-538)
    within the north-star 2e-3, and the exact product of the operands the
    kernel forms -- q * fp16(fp16(x) * fp16(scale * 2^e)) on the fast path,
    q * fp32(fp16(x) * scale * 2^e) on the fp32 path -- within 1e-6 (fp64
    summation order only).
"""

import ctypes
import os

import numpy as np
import pytest

import inputs
from oracle import mtc_oracle as O
from strip_emul import emulated_product

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
MODES = (2, 3, 4, 5, 6, 8)


@pytest.fixture(scope="module")
def model():
    from tensorpack_b200 import build

    build.build()
    path = build.build_strip_model()
    lib = ctypes.CDLL(path)
    lib.strip_model_gemm.restype = ctypes.c_int
    lib.strip_model_gemm.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_int] * 5 + [ctypes.c_void_p, ctypes.c_int] + \
        [ctypes.c_void_p] * 3 + [ctypes.c_uint32]
    lib.strip_model_lane_roundtrip.restype = ctypes.c_int
    lib.strip_model_lane_roundtrip.argtypes = [ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
    return lib


def _roundtrip(model, cls, q):
    q = np.ascontiguousarray(q, dtype=np.int32)
    out = np.zeros(16, np.int32)
    words = np.zeros(5, np.uint32)
    rc = model.strip_model_lane_roundtrip(cls, q.ctypes.data, out.ctypes.data, words.ctypes.data)
    return rc, out, words


@pytest.mark.parametrize("cls", range(6))
def test_lane_codes_roundtrip(model, cls):
    m = MODES[cls]
    lo, hi = -(1 << (m - 1)), (1 << (m - 1)) - 1
    rng = np.random.default_rng(cls)
    cases = [np.full(16, lo), np.full(16, hi), np.arange(16) % (hi - lo + 1) + lo]
    cases += [rng.integers(lo, hi + 1, 16) for _ in range(200)]
    for q in cases:
        rc, out, _ = _roundtrip(model, cls, q)
        assert rc == 0, f"P{m}: placement collision"
        assert np.array_equal(out, q), (m, q, out)
    # every code bit has its own position: all-ones codes set exactly 16 m bits
    _, _, words = _roundtrip(model, cls, np.full(16, hi))  # u = 2^m - 1
    bits = sum(bin(int(w)).count("1") for w in words)
    assert bits == 16 * m


def _check(model, mat, deq_orig, X, tol_emul=1e-6, wide=False, merge=False):
    from tensorpack_b200.core import strip

    hs = strip.build_host(mat, wide=wide, merge_modes=merge)
    # structure of the batch records
    offs = hs.batch_off.astype(np.int64)
    assert (offs % 16 == 0).all() and (np.diff(offs) >= 16).all()
    assert np.diff(offs).max() == hs.max_batch_bytes <= strip.BATCH_BYTES
    assert offs[-1] <= hs.stream.size
    sb = hs.strip_batch.astype(np.int64)
    assert sb[0] == 0 and sb[-1] == hs.n_batches and (np.diff(sb) >= 1).all()
    assert hs.n_strips == 4 * hs.tn
    K, N = mat.shape
    M = X.shape[0]
    pr = None if mat.row_perm is None else np.ascontiguousarray(mat.row_perm, dtype=np.int32)
    pc = None if mat.col_perm is None else np.ascontiguousarray(mat.col_perm, dtype=np.int32)
    Y = np.zeros((M, N), np.float32)
    Xc = np.ascontiguousarray(X, dtype=np.float32)
    rc = model.strip_model_gemm(hs.stream.ctypes.data, hs.batch_off.ctypes.data, hs.strip_batch.ctypes.data,
                                hs.n_strips, hs.tk, K, N, hs.exp2, Xc.ctypes.data, M,
                                None if pr is None else pr.ctypes.data, None if pc is None else pc.ctypes.data,
                                Y.ctypes.data, hs.flags)
    assert rc == 0
    ref = X.astype(np.float64) @ deq_orig.astype(np.float64)
    assert O.relative_frobenius_error(ref, Y) < 2e-3
    emul, fast = emulated_product(mat, deq_orig, X, hs.exp2)
    assert O.relative_frobenius_error(emul, Y) < tol_emul
    return hs, fast


def _qt(golden, name, prefix):
    g = np.load(os.path.join(golden, name))
    sizes = tuple(int(s) for s in g[prefix + "sizes"])
    return g, O.QuadtreeAllocation(sizes, {s: g[f"{prefix}leaf_{s}"] for s in sizes},
                                   {s: g[f"{prefix}modes_{s}"] for s in sizes},
                                   {s: g[f"{prefix}scales_{s}"] for s in sizes}, None,
                                   int(g[prefix + "total_bits"]))


@pytest.mark.parametrize("wide", [False, True])
@pytest.mark.parametrize("M", [1, 2, 3, 4])
def test_forced_modes_all_edges(model, M, wide):
    """All eight precisions at all four leaf edges, signed bf16 scales."""
    from tensorpack_b200.kernels.gemm import MTCMatrix

    W, sizes, leaf, modes, scales = inputs.forced_mode_allocation(256, 384, seed=0, p_split=0.5)
    alloc = O.QuadtreeAllocation(sizes, leaf, modes, scales, None, 0)
    deq = O.quadtree_dequant(W, sizes, leaf, modes, scales)
    m = MTCMatrix.from_qt_allocation(W, alloc)
    X = np.random.default_rng(M).standard_normal((M, 256)).astype(np.float32)
    hs, fast = _check(model, m, deq, X, wide=wide)
    assert (~fast).any() and fast.any()  # both the fast and the fp32 path ran


@pytest.mark.parametrize("wide", [False, True])
@pytest.mark.parametrize("M", [1, 4])
def test_llm_like_permuted(model, golden_dir, M, wide):
    from tensorpack_b200.kernels.gemm import MTCMatrix

    g, inner = _qt(golden_dir, "llm_like_256x512.npz", "b4.25_inner_")
    W, _ = inputs.llm_like(256, 512, seed=1)
    pr, pc = g["b4.25_row_perm"], g["b4.25_col_perm"]
    m = MTCMatrix.from_qt_allocation(W, O.PermutedAllocation(inner, pr, pc, None, int(g["b4.25_total_bits"])))
    stored = O.quadtree_dequant(W[pr][:, pc], inner.sizes, inner.leaf, inner.modes, inner.scales)
    X = inputs.llm_activations(M, 256, seed=M, outlier_seed=1)
    _check(model, m, O.unpermute(stored, pr, pc), X, wide=wide)


@pytest.mark.parametrize("wide", [False, True])
def test_multiscale(model, golden_dir, wide):
    from tensorpack_b200.kernels.gemm import MTCMatrix

    g, a = _qt(golden_dir, "multiscale_256.npz", "")
    W = inputs.multiscale(256, seed=2)
    m = MTCMatrix.from_qt_allocation(W, a)
    deq = O.quadtree_dequant(W, a.sizes, a.leaf, a.modes, a.scales)
    X = np.random.default_rng(0).standard_normal((2, 256)).astype(np.float32)
    _check(model, m, deq, X, wide=wide)


@pytest.mark.parametrize("wide", [False, True])
def test_ragged_fixed_blocks_fp32_scales(model, wide):
    """48 x 80 (padded to 64 x 96), 16x16 blocks of every mode, fp32 scales:
    inexact scales and P16 take the fp32 path, padding strips are empty."""
    from tensorpack_b200.kernels.gemm import MTCMatrix

    rng = np.random.default_rng(3)
    W = rng.standard_normal((48, 80)).astype(np.float32)
    modes = rng.choice([0, 2, 3, 4, 5, 6, 8, 16], size=(3, 5)).astype(np.uint8)
    qmax = np.array([1.0 if x in (0, 2) else 2.0 ** (int(x) - 1) - 1 for x in modes.ravel()]).reshape(3, 5)
    scales = (np.abs(W.reshape(3, 16, 5, 16)).max(axis=(1, 3)) / qmax).astype(np.float32)
    m = MTCMatrix.from_allocation(W, modes, scales, 16)
    deq = O.fixed_dequant(W, modes, np.where(modes == 0, 0, scales).astype(np.float32), 16)
    X = rng.standard_normal((3, 48)).astype(np.float32)
    _check(model, m, deq, X, wide=wide)


def test_all_p0_matrix_gives_zeros(model):
    from tensorpack_b200.kernels.gemm import MTCMatrix

    W = np.zeros((64, 64), np.float32)
    m = MTCMatrix.from_allocation(W, np.zeros((4, 4), np.uint8), np.zeros((4, 4), np.float32), 16)
    X = np.ones((1, 64), np.float32)
    hs, _ = _check(model, m, np.zeros((64, 64), np.float32), X)
    assert hs.n_batches == hs.n_strips  # one empty record per strip


def test_stream_bytes_near_accounted(golden_dir):
    """Decode reads the stream once: its size stays close to the accounted bits."""
    from tensorpack_b200.core import strip
    from tensorpack_b200.kernels.gemm import MTCMatrix

    g, inner = _qt(golden_dir, "llm_like_256x512.npz", "b4.25_inner_")
    W, _ = inputs.llm_like(256, 512, seed=1)
    pr, pc = g["b4.25_row_perm"], g["b4.25_col_perm"]
    m = MTCMatrix.from_qt_allocation(W, O.PermutedAllocation(inner, pr, pc, None, int(g["b4.25_total_bits"])))
    hs = strip.build_host(m)
    ratio = int(hs.batch_off[-1]) / (m.accounted_bits / 8)
    assert ratio < 1.25, ratio


@pytest.mark.parametrize("n_cta,n_warps", [(1, 1), (5, 16), (13, 4), (64, 16), (148, 16), (400, 24)])
def test_schedule_covers_and_balances(golden_dir, n_cta, n_warps):
    """The static schedule hands every batch record to exactly one warp,
    each warp's items are one strip after another, the flush bit closes
    every segment with its own slot, and each CTA's reduction table lists
    its strips with the slot ranges of their segments in order."""
    from tensorpack_b200.core import strip
    from tensorpack_b200.kernels.gemm import MTCMatrix

    g, inner = _qt(golden_dir, "llm_like_256x512.npz", "b4.25_inner_")
    W, _ = inputs.llm_like(256, 512, seed=1)
    pr, pc = g["b4.25_row_perm"], g["b4.25_col_perm"]
    m = MTCMatrix.from_qt_allocation(W, O.PermutedAllocation(inner, pr, pc, None, int(g["b4.25_total_bits"])))
    hs = strip.build_host(m, batch_bytes=2048)
    sc = hs.schedule(n_cta, n_warps)
    n_cta = min(n_cta, hs.n_strips)
    assert sc.n_cta == n_cta and sc.warp_work.size == n_cta * n_warps + 1
    assert sc.warp_work[0] == 0 and sc.warp_work[-1] == hs.n_batches and (np.diff(sc.warp_work.astype(np.int64)) >= 0).all()
    off = sc.work[0::2].astype(np.int64)
    w1 = sc.work[1::2].astype(np.int64)
    nbytes, slot, flush = (w1 & 0xFFF) << 4, (w1 >> 12) & 0x7FFFF, w1 >> 31
    bo = hs.batch_off.astype(np.int64)
    batch_of = {int(o): b for b, o in enumerate(bo[:-1])}
    batches = np.array([batch_of[int(o)] for o in off])
    assert np.array_equal(np.sort(batches), np.arange(hs.n_batches))       # every record exactly once
    assert np.array_equal(nbytes, bo[batches + 1] - bo[batches])
    strip_of = np.searchsorted(hs.strip_batch.astype(np.int64), batches, side="right") - 1
    assert sc.cta_red[0] == 0 and sc.cta_red[-1] == hs.n_strips
    seen = np.zeros(hs.n_strips, np.int64)
    for c in range(n_cta):
        items = range(int(sc.warp_work[c * n_warps]), int(sc.warp_work[(c + 1) * n_warps]))
        red = sc.red.reshape(-1, 3)[sc.cta_red[c]:sc.cta_red[c + 1]]
        seen[red[:, 0]] += 1
        expect = {}
        for w in range(n_warps):
            lo, hi = int(sc.warp_work[c * n_warps + w]), int(sc.warp_work[c * n_warps + w + 1])
            for i in range(lo, hi):
                last = i + 1 == hi or strip_of[i + 1] != strip_of[i]
                assert flush[i] == (1 if last else 0)
                if last:
                    expect.setdefault(int(strip_of[i]), []).append(int(slot[i]))
                if i > lo and strip_of[i] == strip_of[i - 1]:
                    assert slot[i] == slot[i - 1] and batches[i] == batches[i - 1] + 1
        got = {int(s): list(range(int(f), int(f) + int(n))) for s, f, n in red}
        assert got == expect
        slots = [x for v in expect.values() for x in v]
        assert sorted(slots) == list(range(len(slots))) and len(slots) <= sc.max_slots
        assert set(int(s) for s in strip_of[list(items)]) == set(got)
    assert (seen == 1).all()


def test_schedule_rejects_bad_sizes():
    from tensorpack_b200.core import strip

    hs = _llm_host()
    with pytest.raises(ValueError, match="bad sizes"):
        hs.schedule(1, 0)
    with pytest.raises(ValueError, match="bad sizes"):
        hs.schedule(1, 33)


def _llm_host(batch_bytes=2048):
    from tensorpack_b200.core import strip
    from tensorpack_b200.kernels.gemm import MTCMatrix

    g, inner = _qt(os.path.join(ROOT, "tests", "golden"), "llm_like_256x512.npz", "b4.25_inner_")
    W, _ = inputs.llm_like(256, 512, seed=1)
    pr, pc = g["b4.25_row_perm"], g["b4.25_col_perm"]
    m = MTCMatrix.from_qt_allocation(W, O.PermutedAllocation(inner, pr, pc, None, int(g["b4.25_total_bits"])))
    return strip.build_host(m, batch_bytes=batch_bytes)


@pytest.mark.parametrize("damage", ["strip", "nsteps", "kind", "count", "size", "run", "row", "offset", "cover"])
def test_validator_rejects_damaged_streams(damage):
    """mtc_strip_check, which gates every upload, names the first bad record."""
    import copy

    from tensorpack_b200.core import strip

    hs = _llm_host()
    bad = copy.deepcopy(hs)
    o = int(bad.batch_off[3])
    words = bad.stream[o:o + 64].view(np.uint32)  # header + descriptors of batch 3
    if damage == "strip":
        words[0] += 1
    elif damage == "nsteps":
        words[1] = 10 ** 6
    elif damage == "kind":
        words[2] = (words[2] & ~np.uint32(15)) | np.uint32(13)
    elif damage == "count":
        words[2] = (words[2] & ~np.uint32(31 << 5)) | np.uint32(9 << 5)
    elif damage == "size":
        words[2] = words[2] + np.uint32(1 << 15)
    elif damage == "run":
        words[2] = (words[2] & np.uint32(0x3FFFFF)) | np.uint32(1000 << 22)
    elif damage == "row":
        nst = int(words[1])
        st = o + ((8 + 4 * nst + 15) // 16) * 16
        bad.stream[st + 2:st + 4] = 0xFF  # first entry's k row
    elif damage == "offset":
        bad.batch_off[5] += 16
    elif damage == "cover":
        bad.strip_batch[-1] -= 1
    with pytest.raises(ValueError, match="strip stream"):
        strip.check(bad)
    strip.check(hs)  # the undamaged stream passes


def test_decode_rejects_bad_arguments_without_a_gpu():
    """Argument and schedule checks come before any CUDA call."""
    import ctypes

    from tensorpack_b200 import _lib

    lib = _lib.load()
    hs = _llm_host()
    sc = hs.schedule(4)
    d = hs.desc(16, 16, 16, sc, [16, 16, 16, 16])  # fake device pointers: nothing is launched
    X = Y = 16

    def call(desc, M=1, ldx=256, ldy=512):
        return lib.mtc_strip_decode(ctypes.byref(desc), X, M, ldx, None, None, Y, ldy, None, None, None)

    for M in (0, 5):
        assert call(d, M=M) == _lib.MTC_ERR_INVALID and b"M=" in lib.mtc_last_error()
    assert call(d, ldx=255) == _lib.MTC_ERR_INVALID
    bad = _lib.StripDesc.from_buffer_copy(d)
    bad.n_cta = 0
    assert call(bad) == _lib.MTC_ERR_INVALID and b"schedule" in lib.mtc_last_error()
    bad = _lib.StripDesc.from_buffer_copy(d)
    bad.n_warps = 40
    assert call(bad) == _lib.MTC_ERR_INVALID and b"schedule" in lib.mtc_last_error()
    bad = _lib.StripDesc.from_buffer_copy(d)
    bad.max_cta_slots = 0
    assert call(bad) == _lib.MTC_ERR_INVALID and b"max_cta_slots" in lib.mtc_last_error()
    bad = _lib.StripDesc.from_buffer_copy(d)
    bad.work = None
    assert call(bad) == _lib.MTC_ERR_INVALID and b"null" in lib.mtc_last_error()
    bad = _lib.StripDesc.from_buffer_copy(d)
    bad.stream = 8  # not 16-byte aligned
    assert call(bad) == _lib.MTC_ERR_INVALID
    bad = _lib.StripDesc.from_buffer_copy(d)
    bad.flags = 6  # unknown stream flags
    assert call(bad) == _lib.MTC_ERR_INVALID and b"flags" in lib.mtc_last_error()


def test_wide_stream_packs_sixteen_groups_per_step(golden_dir):
    """Wide streams fill group steps with up to 16 groups, are as compact as
    the narrow form, and pass the validator only with their own flag."""
    from tensorpack_b200 import _lib
    from tensorpack_b200.core import strip
    from tensorpack_b200.kernels.gemm import MTCMatrix

    g, inner = _qt(golden_dir, "llm_like_256x512.npz", "b4.25_inner_")
    W, _ = inputs.llm_like(256, 512, seed=1)
    pr, pc = g["b4.25_row_perm"], g["b4.25_col_perm"]
    m = MTCMatrix.from_qt_allocation(W, O.PermutedAllocation(inner, pr, pc, None, int(g["b4.25_total_bits"])))
    narrow, wide = strip.build_host(m), strip.build_host(m, wide=True)
    assert wide.flags == _lib.STRIP_WIDE and narrow.flags == 0
    assert abs(int(wide.batch_off[-1]) - int(narrow.batch_off[-1])) < 0.02 * int(narrow.batch_off[-1])
    n_max = 0
    for b in range(wide.n_batches):
        o = int(wide.batch_off[b])
        nst = int(wide.stream[o + 4:o + 8].view(np.uint32)[0])
        d = wide.stream[o + 8:o + 8 + 4 * nst].view(np.uint32)
        grp = (d & 15) < 6
        if grp.any():
            n_max = max(n_max, int(((d[grp] >> 5) & 31).max()))
    assert n_max == 16
    import copy

    relabeled = copy.deepcopy(wide)
    relabeled.flags = 0
    with pytest.raises(ValueError):
        strip.check(relabeled)


@pytest.mark.parametrize("wide", [False, True])
def test_merged_modes_are_exact_and_drop_p2_p6_kinds(model, wide):
    """P2 items packed with the P3 decoder and P6 items with the P8 one give
    the same product, and the stream then has no P2 / P6 steps."""
    from tensorpack_b200.core import strip
    from tensorpack_b200.kernels.gemm import MTCMatrix

    W, sizes, leaf, modes, scales = inputs.forced_mode_allocation(256, 384, seed=0, p_split=0.5)
    alloc = O.QuadtreeAllocation(sizes, leaf, modes, scales, None, 0)
    deq = O.quadtree_dequant(W, sizes, leaf, modes, scales)
    m = MTCMatrix.from_qt_allocation(W, alloc)
    X = np.random.default_rng(5).standard_normal((2, 256)).astype(np.float32)
    hs, _ = _check(model, m, deq, X, wide=wide, merge=True)
    kinds = set()
    for b in range(hs.n_batches):
        o = int(hs.batch_off[b])
        nst = int(hs.stream[o + 4:o + 8].view(np.uint32)[0])
        kinds |= set((hs.stream[o + 8:o + 8 + 4 * nst].view(np.uint32) & 15).tolist())
    assert not kinds & {0, 4, 6, 10} and kinds & {1, 5, 7, 11}  # no G2, G6, U2, U6; merged kinds present


@pytest.mark.parametrize("wide", [False, True])
def test_shape_not_multiple_of_eight(model, wide):
    """44 x 84 in 4x4 blocks of every mode: the last strip straddles N (its
    columns beyond 84 are padding) and K is padded to 64."""
    from tensorpack_b200.kernels.gemm import MTCMatrix

    rng = np.random.default_rng(11)
    W = rng.standard_normal((44, 84)).astype(np.float32)
    modes = rng.choice([0, 2, 3, 4, 5, 6, 8, 16], size=(11, 21)).astype(np.uint8)
    qmax = np.array([1.0 if x in (0, 2) else 2.0 ** (int(x) - 1) - 1 for x in modes.ravel()]).reshape(11, 21)
    amax = np.abs(W.reshape(11, 4, 21, 4)).max(axis=(1, 3))
    scales = (amax / qmax).astype(np.float32)
    scales = (scales.view(np.uint32) & 0xFFFF0000).view(np.float32)  # bf16 scales: the fast path
    m = MTCMatrix.from_allocation(W, modes, scales, 4)
    deq = O.fixed_dequant(W, modes, np.where(modes == 0, 0, scales).astype(np.float32), 4)
    X = rng.standard_normal((2, 44)).astype(np.float32)
    _check(model, m, deq, X, wide=wide)


@pytest.mark.parametrize("wide", [False, True])
def test_runs_of_full_steps(model, wide):
    """A 1024-row LLM-like layer (oracle allocation, MTC-QT-P at 4.25 b/w)
    gives runs of identical full steps in both forms; the kernel's counted
    run loop is checked through the model."""
    from tensorpack_b200.core import strip
    from tensorpack_b200.kernels.gemm import MTCMatrix

    W, h = inputs.llm_like(1024, 128, seed=3)
    a = O.PermutedQuadtree(W, h, sizes=(32, 16, 8, 4)).select(4.25)
    m = MTCMatrix.from_qt_allocation(W, a)
    hs = strip.build_host(m, wide=wide)
    runs = 0
    for b in range(hs.n_batches):
        o = int(hs.batch_off[b])
        nst = int(hs.stream[o + 4:o + 8].view(np.uint32)[0])
        runs += int(((hs.stream[o + 8:o + 8 + 4 * nst].view(np.uint32) >> 22) > 1).sum())
    assert runs > 0
    X = inputs.llm_activations(2, 1024, seed=4, outlier_seed=0)
    _check(model, m, a.dequant, X, wide=wide)


def test_strip_exp2_edge_cases():
    """The pre-scale puts the largest |scale| of a live leaf in (1/2, 1];
    matrices with no live scale use 0; extreme scales are clamped."""
    from tensorpack_b200.core import layout, strip

    def ls(modes, scales):
        n = len(modes)
        z = np.zeros(n, np.int64)
        return layout.LeafSet(z, z, np.full(n, 4), np.asarray(modes, np.uint8), np.asarray(scales, np.float32), z)

    assert strip.strip_exp2(ls([0, 0], [5.0, 7.0])) == 0            # P0 leaves only
    assert strip.strip_exp2(ls([4, 4], [0.0, 0.0])) == 0            # zero scales only
    for smax in (0.75, 1.0, 3.0, 1e-3, -40.0):
        e = strip.strip_exp2(ls([4, 0, 8], [smax, 1e6, smax / 3]))  # the P0 leaf's scale is ignored
        assert 0.5 < abs(smax) * 2.0 ** e <= 1.0, (smax, e)
    assert strip.strip_exp2(ls([4], [1e-38])) == 100                # clamped


def test_strip_fits_shared_memory_limits():
    """The host-side query mirrors the launch plan: the gathered activations
    (M x K fp16) must fit next to the batch slots."""
    import ctypes

    from tensorpack_b200 import _lib

    lib = _lib.load()
    hs = _llm_host()
    d = hs.desc(16, 16, 16, hs.schedule(4), [16, 16, 16, 16])
    for M in (1, 2, 3, 4):
        assert lib.mtc_strip_fits(ctypes.byref(d), M) == 1
    assert lib.mtc_strip_fits(ctypes.byref(d), 0) == 0 and lib.mtc_strip_fits(ctypes.byref(d), 5) == 0
    big = _lib.StripDesc.from_buffer_copy(d)
    big.tk = 28672 // 32  # Llama-70B down_proj K
    assert lib.mtc_strip_fits(ctypes.byref(big), 1) == 1
    assert lib.mtc_strip_fits(ctypes.byref(big), 4) == 0   # 4 x 28672 fp16 rows do not fit with the slots
    big.tk = 200000 // 32
    assert lib.mtc_strip_fits(ctypes.byref(big), 1) == 0
