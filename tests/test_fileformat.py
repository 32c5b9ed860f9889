"""On-disk format of packed matrices (tensorpack_b200.core.fileformat), CPU only.

Round trips of the reference's fixed-block layout and of MTC-QT-P quadtree
matrices must restore every byte of the host layout (arena, offsets, modes,
scales, leaf placement, permutations) and the same accounted size; the
committed version-1 fixture pins the container format; corrupt, truncated or
foreign files and inconsistent matrices are rejected with ValueError.
"""

import json
import os
import struct

import numpy as np
import pytest

import inputs
from oracle import mtc_oracle as O
from tensorpack_b200.core import fileformat as F
from tensorpack_b200.kernels import device as D
from tensorpack_b200.kernels.gemm import MTCMatrix
from test_host_layout import decode_arena, load, qt_from_golden


def same_host_layout(a: MTCMatrix, b: MTCMatrix):
    assert a.shape == b.shape and a.block_size == b.block_size and a.sizes == b.sizes
    assert a.total_bytes_allocated == b.total_bytes_allocated
    n = a.total_bytes_allocated
    np.testing.assert_array_equal(a.arena.raw_buffer[:n], b.arena.raw_buffer[:n])
    for f in ("offsets", "precisions", "scales", "leaf_rows", "leaf_cols", "leaf_sizes", "row_perm", "col_perm"):
        x, y = getattr(a, f), getattr(b, f)
        assert (x is None) == (y is None), f
        if x is not None:
            np.testing.assert_array_equal(np.asarray(x), np.asarray(y), err_msg=f)
    assert a.accounted_bits == b.accounted_bits
    assert a.average_bits_per_element == b.average_bits_per_element
    assert a.scale_format == b.scale_format


def fixed_matrix(golden_dir):
    g = load(golden_dir, "fixed_pair.npz")
    A, _ = inputs.fixed_pair(seed=5)
    return MTCMatrix.from_allocation(A, g["b5.2_A_modes"], g["b5.2_A_scales"], 16), g


def qtp_matrix(golden_dir):
    g = load(golden_dir, "llm_like_256x512.npz")
    W, _ = inputs.llm_like(256, 512, seed=1)
    inner = qt_from_golden(g, "b4.25_inner_")
    alloc = O.PermutedAllocation(inner, g["b4.25_row_perm"], g["b4.25_col_perm"], None, int(g["b4.25_total_bits"]))
    return MTCMatrix.from_qt_allocation(W, alloc), alloc, W


def test_fixed_block_round_trip(golden_dir, tmp_path):
    m, g = fixed_matrix(golden_dir)
    p = tmp_path / "fixed.mtcpk"
    m.save(p)
    r = MTCMatrix.load(p)
    same_host_layout(m, r)
    assert not r.is_quadtree and r.num_blocks == m.num_blocks
    np.testing.assert_array_equal(decode_arena(r), g["b5.2_A_dequant"])


@pytest.mark.parametrize("mmap", [False, True])
def test_permuted_quadtree_round_trip(golden_dir, tmp_path, mmap):
    m, alloc, W = qtp_matrix(golden_dir)
    p = tmp_path / "qtp.mtcpk"
    m.save(p)
    r = MTCMatrix.load(p, mmap=mmap)
    same_host_layout(m, r)
    assert r.is_quadtree and r.accounted_bits == alloc.total_bits
    ref = O.permuted_quadtree_dequant(W, alloc.row_perm, alloc.col_perm, alloc.inner.sizes, alloc.inner.leaf,
                                      alloc.inner.modes, alloc.inner.scales)
    np.testing.assert_array_equal(O.unpermute(decode_arena(r), r.row_perm, r.col_perm), ref)
    # bf16-exact scales are stored as 16-bit words, as the accounted format counts them
    assert "scales_bf16" in F.read_header(p)["entries"]["matrix"]["arrays"]


def test_bundle_of_named_matrices(golden_dir, tmp_path):
    m1, _ = fixed_matrix(golden_dir)
    m2, _, _ = qtp_matrix(golden_dir)
    p = tmp_path / "model.mtcpk"
    F.save_mtc(p, {"layers.0.gate": m2, "layers.0.down": m1})
    out = F.load_mtc(p)
    assert sorted(out) == ["layers.0.down", "layers.0.gate"]
    same_host_layout(out["layers.0.gate"], m2)
    same_host_layout(out["layers.0.down"], m1)
    with pytest.raises(ValueError, match="bundle"):
        MTCMatrix.load(p)
    with pytest.raises(ValueError, match="name"):
        F.save_mtc(tmp_path / "bad.mtcpk", {"a/b": m1})


def test_version1_fixture_is_pinned(golden_dir, tmp_path):
    """The committed fixture loads with this reader, decodes to the oracle's
    dequant of the allocation it was made from, and saving it again gives
    byte-identical output (the writer is deterministic)."""
    import make_pack_fixture

    W, alloc, ref_m = make_pack_fixture.fixture_matrix()
    path = os.path.join(golden_dir, "pack_v1.mtcpk")
    m = MTCMatrix.load(path)
    same_host_layout(m, ref_m)
    assert m.scale_format == "fp32"
    assert set(np.unique(m.precisions).tolist()) == {0, 2, 3, 4, 5, 6, 8, 16}
    assert set(np.unique(m.leaf_sizes).tolist()) == {4, 8, 16, 32}
    ref = O.permuted_quadtree_dequant(W, alloc.row_perm, alloc.col_perm, alloc.inner.sizes, alloc.inner.leaf,
                                      alloc.inner.modes, alloc.inner.scales)
    np.testing.assert_array_equal(O.unpermute(decode_arena(m), m.row_perm, m.col_perm), ref)
    again = tmp_path / "again.mtcpk"
    m.save(again)
    assert open(path, "rb").read() == open(again, "rb").read()


def _rewrite(path, fn):
    b = bytearray(open(path, "rb").read())
    fn(b)
    open(path, "wb").write(bytes(b))


def test_corrupt_truncated_and_foreign_files_rejected(golden_dir, tmp_path):
    m, _, _ = qtp_matrix(golden_dir)
    p = tmp_path / "x.mtcpk"
    m.save(p)
    good = open(p, "rb").read()
    h = F.read_header(p)
    arena_off = h["entries"]["matrix"]["arrays"]["arena"]["offset"]

    def flip(b):
        b[arena_off + 17] ^= 0x40

    _rewrite(p, flip)
    with pytest.raises(ValueError, match="checksum"):
        MTCMatrix.load(p)
    open(p, "wb").write(good[:len(good) - 100])
    with pytest.raises(ValueError, match="outside the file|truncated"):
        MTCMatrix.load(p)
    open(p, "wb").write(b"NOTMTC\0\0" + good[8:])
    with pytest.raises(ValueError, match="magic"):
        MTCMatrix.load(p)
    open(p, "wb").write(good[:8] + struct.pack("<I", 99) + good[12:])
    with pytest.raises(ValueError, match="version"):
        MTCMatrix.load(p)
    open(p, "wb").write(good[:10])
    with pytest.raises(ValueError, match="too short"):
        MTCMatrix.load(p)


def _save_raw(path, m):
    """Save without the writer's checks (the matrix may be inconsistent)."""
    F.save_mtc(path, m)


def test_inconsistent_matrices_rejected(golden_dir, tmp_path):
    m, _, _ = qtp_matrix(golden_dir)
    p = tmp_path / "bad.mtcpk"
    # two leaves swapped in place: the same area, but a gap and an overlap
    rows = np.asarray(m.leaf_rows).copy()
    sizes = np.asarray(m.leaf_sizes)
    i = int(np.nonzero(sizes == 4)[0][0])
    j = int(np.nonzero((sizes == 4) & (np.arange(len(sizes)) != i))[0][0])
    rows[i] = rows[j]
    cols = np.asarray(m.leaf_cols).copy()
    cols[i] = cols[j]
    bad = MTCMatrix(m.shape, m.block_size, m.arena, m.offsets, m.precisions, m.scales, None, leaf_rows=rows,
                    leaf_cols=cols, leaf_sizes=m.leaf_sizes, sizes=m.sizes, row_perm=m.row_perm, col_perm=m.col_perm)
    _save_raw(p, bad)
    with pytest.raises(ValueError, match="cover"):
        MTCMatrix.load(p)
    # a row permutation with a repeated index
    rp = np.asarray(m.row_perm).copy()
    rp[0] = rp[1]
    bad = MTCMatrix(m.shape, m.block_size, m.arena, m.offsets, m.precisions, m.scales, None,
                    leaf_rows=m.leaf_rows, leaf_cols=m.leaf_cols, leaf_sizes=m.leaf_sizes, sizes=m.sizes,
                    row_perm=rp, col_perm=m.col_perm)
    _save_raw(p, bad)
    with pytest.raises(ValueError, match="permutation"):
        MTCMatrix.load(p)
    # a payload offset past the end of the arena
    offs = np.asarray(m.offsets).copy()
    live = int(np.nonzero(np.asarray(m.precisions) != 0)[0][-1])
    offs[live] = m.total_bytes_allocated
    bad = MTCMatrix(m.shape, m.block_size, m.arena, offs, m.precisions, m.scales, None, leaf_rows=m.leaf_rows,
                    leaf_cols=m.leaf_cols, leaf_sizes=m.leaf_sizes, sizes=m.sizes, row_perm=m.row_perm,
                    col_perm=m.col_perm)
    _save_raw(p, bad)
    with pytest.raises(ValueError, match="arena"):
        MTCMatrix.load(p)


def _fake_stream(tk=3, tn=10):
    """Consistent stream buffers of the sizes the device format uses."""
    nb = -(-tn // D.BAND_TILES)
    n_sub = 2 * nb * ((tk + 1) // 2)
    sizes = (np.arange(n_sub, dtype=np.int64) % 5 + 9) * 16
    offs = np.concatenate([[0], np.cumsum(sizes)]).astype(np.uint32).view(np.int32)
    ranges = np.zeros((n_sub, 4), np.uint32)
    ranges[:, 0] = sizes
    rb = 4096
    row_off = np.tile(np.linspace(0, rb, tk + 1).astype(np.int32), nb)
    meta = {"version": D.STREAM_FORMAT_VERSION, "band_tiles": D.BAND_TILES, "K": 32 * tk, "N": 32 * tn, "tk": tk,
            "tn": tn, "exp2": 0, "scale_words": 1, "record_bytes": rb, "max_row_bytes": 2048,
            "max_stage_bytes": int(sizes.max())}
    arrs = {"tiles": np.zeros(tk * tn * 16, np.uint8), "row_off": row_off, "records": np.zeros(rb, np.uint8),
            "stage_counts": np.zeros(n_sub, np.int32), "stage_offsets": offs,
            "stage_ranges": ranges.reshape(-1).view(np.int32), "stage_images": np.zeros(int(sizes.sum()), np.uint8)}
    return meta, arrs


def test_saved_stream_checks():
    meta, arrs = _fake_stream()
    D.check_stream_buffers(meta, arrs)
    bad = dict(arrs, stage_images=arrs["stage_images"][:-16])
    with pytest.raises(ValueError, match="outside"):
        D.check_stream_buffers(meta, bad)
    ro = arrs["row_off"].copy()
    ro[1] = 5000
    with pytest.raises(ValueError, match="row offsets"):
        D.check_stream_buffers(meta, dict(arrs, row_off=ro))
    with pytest.raises(ValueError, match="tiles"):
        D.check_stream_buffers(meta, dict(arrs, tiles=arrs["tiles"][:-1]))
    with pytest.raises(ValueError, match="maximum"):
        D.check_stream_buffers(dict(meta, max_stage_bytes=16), arrs)
    offs = arrs["stage_offsets"].copy()
    offs[1] += 16
    with pytest.raises(ValueError, match="overlap"):
        D.check_stream_buffers(meta, dict(arrs, stage_offsets=offs))


def test_stream_compatibility_rules(golden_dir):
    m, _, _ = qtp_matrix(golden_dir)
    from tensorpack_b200.core import layout

    K, N = m.shape
    meta = {"version": D.STREAM_FORMAT_VERSION, "band_tiles": D.BAND_TILES, "K": K, "N": N, "tk": K // 32,
            "tn": N // 32, "exp2": layout.choose_exp2(m.leaf_set), "scale_words": 1}
    assert D.stream_compatible(meta, m)
    assert not D.stream_compatible(dict(meta, version=D.STREAM_FORMAT_VERSION - 1), m)
    assert not D.stream_compatible(dict(meta, exp2=meta["exp2"] + 1), m)
    assert not D.stream_compatible(dict(meta, N=N + 32), m)
    assert not D.stream_compatible({}, m)


def test_header_is_plain_json(golden_dir, tmp_path):
    m, _ = fixed_matrix(golden_dir)
    p = tmp_path / "h.mtcpk"
    m.save(p)
    raw = open(p, "rb").read()
    magic, ver, hlen, data_off = struct.unpack("<8sIIQ", raw[:24])
    assert magic == b"MTCPACK\0" and ver == 1 and data_off % 64 == 0
    h = json.loads(raw[24:24 + hlen])
    e = h["entries"]["matrix"]
    assert e["kind"] == "fixed" and e["shape"] == list(m.shape) and e["accounted_bits"] == m.accounted_bits
    for rec in e["arrays"].values():
        assert rec["offset"] % 64 == 0 and rec["offset"] >= data_off


def test_strip_stream_saved_and_reused(golden_dir, tmp_path):
    """include_strip stores the decode layout (built on the host, no GPU);
    loading validates it and attaches it, so the decode does not rebuild it."""
    from tensorpack_b200.core import strip

    m = qtp_matrix(golden_dir)[0]
    p = tmp_path / "strip.mtcpk"
    m.save(p, include_strip=True)
    meta = F.read_header(p)["entries"]["matrix"]
    assert meta["strip"]["version"] == strip.STRIP_FORMAT_VERSION
    r = MTCMatrix.load(p)
    same_host_layout(m, r)
    hs, fresh = r.__dict__.get("_host_strip"), strip.build_host(r)
    assert hs is not None, "the saved strip stream was not attached"
    for k in ("stream", "batch_off", "strip_batch"):
        assert np.array_equal(getattr(hs, k), getattr(fresh, k)), k
    assert (hs.exp2, hs.max_batch_bytes, hs.flags) == (fresh.exp2, fresh.max_batch_bytes, fresh.flags)
    # a file without the strip stream loads as before and builds it on demand
    q = tmp_path / "plain.mtcpk"
    m.save(q)
    r2 = MTCMatrix.load(q)
    assert r2.__dict__.get("_host_strip") is None
    assert np.array_equal(r2.host_strip().stream, fresh.stream)


def _save_with_strip(path, m, edit_meta=None, edit_arrays=None):
    """save_mtc with the exported strip stream altered before it is written
    (the file's checksums then match the altered bytes)."""
    from tensorpack_b200.core import strip

    orig = strip.export_host

    def export(hs):
        meta, arrs = orig(hs)
        arrs = {k: v.copy() for k, v in arrs.items()}
        if edit_meta:
            edit_meta(meta)
        if edit_arrays:
            edit_arrays(arrs)
        return meta, arrs

    strip.export_host = export
    try:
        m.save(path, include_strip=True)
    finally:
        strip.export_host = orig


def test_strip_stream_of_another_version_is_rebuilt(golden_dir, tmp_path):
    m = qtp_matrix(golden_dir)[0]
    p = tmp_path / "strip.mtcpk"
    _save_with_strip(p, m, edit_meta=lambda meta: meta.update(version=meta["version"] + 1))
    r = MTCMatrix.load(p)
    assert r.__dict__.get("_host_strip") is None  # ignored, built again on first use


def test_strip_stream_of_another_form_is_rebuilt(golden_dir, tmp_path):
    """A saved wide stream, or one with larger batch records, is not the
    default form: the file loads and the default stream is built again on
    first use instead of failing."""
    from tensorpack_b200 import _lib
    from tensorpack_b200.core import strip

    m = qtp_matrix(golden_dir)[0]
    for name, edit in (("wide", lambda meta: meta.update(flags=_lib.STRIP_WIDE)),
                       ("big", lambda meta: meta.update(max_batch_bytes=2 * strip.BATCH_BYTES))):
        p = tmp_path / f"{name}.mtcpk"
        _save_with_strip(p, m, edit_meta=edit)
        r = MTCMatrix.load(p)
        assert r.__dict__.get("_host_strip") is None, name
        assert np.array_equal(r.host_strip().stream, strip.build_host(r).stream)


def test_damaged_strip_stream_rejected(golden_dir, tmp_path):
    """A strip record that matches its checksum but fails the validator (a
    consistent-looking but wrong file) raises instead of being used."""
    m = qtp_matrix(golden_dir)[0]
    p = tmp_path / "strip.mtcpk"

    def damage(arrs):
        arrs["stream"][0] ^= 0x01  # the strip index of the first batch record

    _save_with_strip(p, m, edit_arrays=damage)
    with pytest.raises(ValueError, match="strip"):
        MTCMatrix.load(p)
