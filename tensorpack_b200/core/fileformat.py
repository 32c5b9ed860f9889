"""Versioned on-disk format of packed MTC matrices (``.mtcpk``).

The reference keeps packed matrices in memory only (mtc/kernels/gemm.py:
217-253 holds the arena, offsets, modes and scales of a live MTCMatrix; the
quadtree and permuted allocations, mtc/core/quadtree.py:55-70 and
mtc/core/permutation.py:54-67, are rebuilt by re-running the allocator).
This module stores everything a packed matrix needs to be used again without
the allocator:

* the host layout: the arena payload bytes (per-mode packing of
  mtc/kernels/gemm.py:457-478), per-leaf offsets, modes and scales (bf16 when
  every scale is bf16-exact, as the accounted format counts them), and for a
  quadtree matrix the leaf placement (row, column, edge) and level sizes;
* the MTC-QT-P row / column permutations;
* optionally the device tile stream (tile descriptors, row offsets, records
  and the sub-stage images of the tensor-core kernels), so that loading onto
  a GPU uploads bytes instead of repacking.  The stream is tagged with the
  device format version; a file whose stream version differs from the
  library's is still loadable, and its stream is rebuilt from the host layout;
* optionally the strip stream of the decode kernel (batch records and their
  tables, built on the host, so saving it needs no GPU), tagged and handled
  the same way: a stream of the library's strip version is validated record
  by record and used instead of being built again.

File layout (little endian):

    0   8 bytes  magic b"MTCPACK\\0"
    8   u32      container version (FORMAT_VERSION)
    12  u32      header length H (bytes of UTF-8 JSON)
    16  u64      offset of the array region (64-byte aligned)
    24  H bytes  JSON header: entries -> {kind, shape, ..., arrays}
    ...          arrays, each starting on a 64-byte boundary

Every array is listed in the header with its dtype, shape, file offset, size
and CRC-32; a reader checks all of them, so truncated or corrupted files
raise ``ValueError`` instead of producing a wrong matrix.  A file holds one
or more named matrices (a bundle: the layers of a model).
"""

from __future__ import annotations

import json
import os
import struct
import zlib
from typing import Dict, Mapping, Optional, Union

import numpy as np

from . import layout
from .arena import MemoryArena
from .types import MODES

MAGIC = b"MTCPACK\0"
FORMAT_VERSION = 1
_ALIGN = 64
_PREFIX = struct.Struct("<8sIIQ")
_SINGLE = "matrix"

PathLike = Union[str, os.PathLike]


def _align(n: int) -> int:
    return (n + _ALIGN - 1) // _ALIGN * _ALIGN


def _small_int(a: np.ndarray, limit: int) -> np.ndarray:
    a = np.asarray(a)
    if a.size and (int(a.min()) < 0 or int(a.max()) > limit):
        raise ValueError("value outside the stored integer range")
    return a


def _host_arrays(mat) -> Dict[str, np.ndarray]:
    """The host layout of one MTCMatrix as named arrays."""
    arrs = {"arena": np.ascontiguousarray(mat.arena.raw_buffer[:mat.total_bytes_allocated])}
    offsets = np.asarray(mat.offsets)
    arrs["offsets"] = _small_int(offsets, 0xFFFFFFFF).astype("<u4")
    arrs["modes"] = np.asarray(mat.precisions).astype("u1")
    scales = np.asarray(mat.scales, dtype=np.float32)
    if layout.bf16_exact(scales):
        arrs["scales_bf16"] = (scales.view(np.uint32) >> 16).astype("<u2")
    else:
        arrs["scales_f32"] = scales.astype("<f4")
    if mat.is_quadtree:
        arrs["leaf_rows"] = _small_int(mat.leaf_rows, 0x7FFFFFFF).astype("<i4")
        arrs["leaf_cols"] = _small_int(mat.leaf_cols, 0x7FFFFFFF).astype("<i4")
        arrs["leaf_sizes"] = _small_int(mat.leaf_sizes, 255).astype("u1")
    if mat.row_perm is not None:
        arrs["row_perm"] = _small_int(mat.row_perm, 0x7FFFFFFF).astype("<i4")
    if mat.col_perm is not None:
        arrs["col_perm"] = _small_int(mat.col_perm, 0x7FFFFFFF).astype("<i4")
    return arrs


def _entry_meta(mat, stream_meta: Optional[dict], strip_meta: Optional[dict] = None) -> dict:
    meta = {
        "kind": "quadtree" if mat.is_quadtree else "fixed",
        "shape": [int(x) for x in mat.shape],
        "block_size": int(mat.block_size),
        "sizes": [int(s) for s in mat.sizes],
        "scale_format": mat.scale_format,
        "accounted_bits": int(mat.accounted_bits),
        "num_leaves": int(mat.num_leaves),
    }
    if stream_meta is not None:
        meta["stream"] = stream_meta
    if strip_meta is not None:
        meta["strip"] = strip_meta
    return meta


def save_mtc(path: PathLike, matrices, *, include_stream: bool = False, device=None,
             include_strip: bool = False) -> None:
    """Write one MTCMatrix, or a mapping name -> MTCMatrix, to ``path``.

    ``include_stream`` also stores each matrix's device tile stream (built on
    ``device``, default the current CUDA device, if it does not exist yet);
    ``include_strip`` stores the strip stream of the decode kernel (built on
    the host)."""
    single = not isinstance(matrices, Mapping)
    items = {_SINGLE: matrices} if single else dict(matrices)
    if not items:
        raise ValueError("nothing to save")
    header = {"format": "mtc-packed", "version": FORMAT_VERSION, "single": single, "entries": {}}
    payload = []  # (array, header record)
    for name, mat in items.items():
        if "/" in name or not name:
            raise ValueError(f"bad matrix name {name!r}")
        arrs = _host_arrays(mat)
        stream_meta = strip_meta = None
        if include_stream:
            ds = mat.device_stream(device)
            stream_meta, sarrs = ds.export_buffers()
            arrs.update({"stream." + k: v for k, v in sarrs.items()})
        if include_strip:
            from . import strip as _strip

            strip_meta, parrs = _strip.export_host(mat.host_strip())
            arrs.update({"strip." + k: v for k, v in parrs.items()})
        recs = {}
        for key, a in arrs.items():
            a = np.ascontiguousarray(a)
            rec = {"dtype": a.dtype.str, "shape": list(a.shape), "nbytes": int(a.nbytes),
                   "crc32": zlib.crc32(a.view(np.uint8).reshape(-1)) & 0xFFFFFFFF}
            recs[key] = rec
            payload.append((a, rec))
        meta = _entry_meta(mat, stream_meta, strip_meta)
        meta["arrays"] = recs
        header["entries"][name] = meta
    # offsets depend on the header length, which depends on the offsets:
    # assign with a fixed-width placeholder, then fill in
    for _, rec in payload:
        rec["offset"] = 0
    while True:
        blob = json.dumps(header, sort_keys=True).encode()
        data_off = _align(_PREFIX.size + len(blob))
        pos, changed = data_off, False
        for a, rec in payload:
            if rec["offset"] != pos:
                rec["offset"], changed = pos, True
            pos = _align(pos + a.nbytes)
        if not changed:
            break
    tmp = os.fspath(path) + ".tmp"
    with open(tmp, "wb") as f:
        f.write(_PREFIX.pack(MAGIC, FORMAT_VERSION, len(blob), data_off))
        f.write(blob)
        for a, rec in payload:
            f.write(b"\0" * (rec["offset"] - f.tell()))
            f.write(a.view(np.uint8).reshape(-1).tobytes())
        f.write(b"\0" * (_align(f.tell()) - f.tell()))
    os.replace(tmp, path)


def read_header(path: PathLike) -> dict:
    """The JSON header of a ``.mtcpk`` file (validates the prefix)."""
    with open(path, "rb") as f:
        pre = f.read(_PREFIX.size)
        if len(pre) < _PREFIX.size:
            raise ValueError(f"{path}: too short for an MTC pack file")
        magic, version, hlen, data_off = _PREFIX.unpack(pre)
        if magic != MAGIC:
            raise ValueError(f"{path}: not an MTC pack file (bad magic)")
        if version != FORMAT_VERSION:
            raise ValueError(f"{path}: container version {version} not supported (this reader: {FORMAT_VERSION})")
        blob = f.read(hlen)
    if len(blob) != hlen:
        raise ValueError(f"{path}: truncated header")
    try:
        header = json.loads(blob.decode())
    except (UnicodeDecodeError, json.JSONDecodeError) as e:
        raise ValueError(f"{path}: corrupt header ({e})") from None
    if header.get("format") != "mtc-packed" or header.get("version") != version:
        raise ValueError(f"{path}: header does not describe an MTC pack")
    if data_off < _PREFIX.size + hlen or data_off % _ALIGN:
        raise ValueError(f"{path}: bad array region offset")
    return header


def _read_arrays(path, recs: dict, mmap: bool, file_size: int) -> Dict[str, np.ndarray]:
    out = {}
    mm = np.memmap(path, dtype=np.uint8, mode="r") if mmap else None
    with open(path, "rb") as f:
        for key, rec in recs.items():
            off, nb = int(rec["offset"]), int(rec["nbytes"])
            dt = np.dtype(rec["dtype"])
            shape = tuple(int(x) for x in rec["shape"])
            if off % _ALIGN or off + nb > file_size or int(np.prod(shape, dtype=np.int64)) * dt.itemsize != nb:
                raise ValueError(f"{path}: array {key!r} lies outside the file or has a bad size")
            if mm is not None:
                raw = mm[off:off + nb]
            else:
                f.seek(off)
                raw = np.frombuffer(f.read(nb), dtype=np.uint8)
                if raw.nbytes != nb:
                    raise ValueError(f"{path}: truncated array {key!r}")
            if (zlib.crc32(raw) & 0xFFFFFFFF) != int(rec["crc32"]):
                raise ValueError(f"{path}: checksum mismatch in array {key!r}")
            out[key] = raw.view(dt).reshape(shape)
    return out


def _check_host(name, meta, a) -> None:
    """Structural checks a packed matrix must pass before any kernel sees it."""
    K, N = meta["shape"]
    modes = a["modes"].reshape(-1)
    n = modes.size
    if not np.isin(modes, MODES).all():
        raise ValueError(f"{name}: unknown precision mode")
    for key in ("offsets",):
        if a[key].size != n:
            raise ValueError(f"{name}: {key} has {a[key].size} entries, modes {n}")
    sc = a.get("scales_bf16", a.get("scales_f32"))
    if sc is None or sc.size != n:
        raise ValueError(f"{name}: scales missing or of the wrong length")
    if meta["kind"] == "quadtree":
        rows, cols, sz = a["leaf_rows"], a["leaf_cols"], a["leaf_sizes"].astype(np.int64)
        if not (rows.size == cols.size == sz.size == n):
            raise ValueError(f"{name}: leaf placement arrays of the wrong length")
        if not np.isin(sz, meta["sizes"]).all():
            raise ValueError(f"{name}: leaf edge not among the quadtree levels")
        if n and ((rows % sz).any() or (cols % sz).any() or (rows < 0).any() or (cols < 0).any()
                  or (rows + sz > K).any() or (cols + sz > N).any()):
            raise ValueError(f"{name}: leaf outside the matrix or not aligned to its edge")
        if int((sz * sz).sum()) != K * N:
            raise ValueError(f"{name}: leaves do not cover the matrix exactly once")
        # exact single coverage on the grid of the smallest leaf edge
        g = int(np.gcd.reduce(np.asarray(meta["sizes"], np.int64))) if n else 1
        if K % g or N % g:
            raise ValueError(f"{name}: shape {K}x{N} is not a multiple of the smallest leaf edge {g}")
        Ng = N // g
        flat = []
        for s in np.unique(sz):
            sel = sz == s
            e = int(s) // g
            offs = (np.arange(e)[:, None] * Ng + np.arange(e)[None, :]).reshape(-1)
            flat.append(((rows[sel] // g) * Ng + cols[sel] // g)[:, None].astype(np.int64) + offs[None, :])
        cover = np.bincount(np.concatenate([f.reshape(-1) for f in flat]), minlength=(K // g) * Ng)
        if cover.size != (K // g) * Ng or (cover != 1).any():
            raise ValueError(f"{name}: leaves do not cover the matrix exactly once")
        edge = sz
    else:
        bs = meta["block_size"]
        if a["modes"].shape != (K // bs, N // bs):
            raise ValueError(f"{name}: block grid {a['modes'].shape} does not match shape {K}x{N}, Bs {bs}")
        edge = np.full(n, bs, np.int64)
    nbytes = modes.astype(np.int64) * edge * edge // 8
    end = a["offsets"].reshape(-1).astype(np.int64) + nbytes
    if n and int(end[modes != 0].max(initial=0)) > a["arena"].size:
        raise ValueError(f"{name}: a leaf payload lies outside the arena")
    for key, length in (("row_perm", K), ("col_perm", N)):
        if key in a:
            p = a[key]
            if p.size != length or not np.array_equal(np.sort(p), np.arange(length)):
                raise ValueError(f"{name}: {key} is not a permutation of {length}")


def _build_matrix(name, meta, a):
    from ..kernels.gemm import MTCMatrix

    _check_host(name, meta, a)
    arena_bytes = a["arena"]
    arena = MemoryArena(capacity_bytes=max(arena_bytes.size, 1))
    base = arena.allocate(arena_bytes.size)
    arena.raw_buffer[base:base + arena_bytes.size] = arena_bytes
    if "scales_bf16" in a:
        scales = (a["scales_bf16"].astype(np.uint32) << 16).view(np.float32)
    else:
        scales = a["scales_f32"].astype(np.float32)
    scales = scales.reshape(a["modes"].shape)
    rp = a["row_perm"].astype(np.int64) if "row_perm" in a else None
    cp = a["col_perm"].astype(np.int64) if "col_perm" in a else None
    if meta["kind"] == "quadtree":
        mat = MTCMatrix(tuple(meta["shape"]), int(meta["block_size"]), arena, a["offsets"].astype(np.uint32),
                        a["modes"].astype(np.uint8).copy(), scales.astype(np.float32).copy(), None,
                        leaf_rows=a["leaf_rows"].astype(np.int64), leaf_cols=a["leaf_cols"].astype(np.int64),
                        leaf_sizes=a["leaf_sizes"].astype(np.int64), sizes=meta["sizes"], row_perm=rp,
                        col_perm=cp)
    else:
        mat = MTCMatrix(tuple(meta["shape"]), int(meta["block_size"]), arena, a["offsets"].astype(np.uint32),
                        a["modes"].astype(np.uint8).copy(), scales.astype(np.float32).copy(), None, row_perm=rp,
                        col_perm=cp)
    if int(mat.accounted_bits) != int(meta["accounted_bits"]):
        raise ValueError(f"{name}: accounted bits {mat.accounted_bits} != recorded {meta['accounted_bits']}")
    return mat


def load_mtc(path: PathLike, *, device=None, use_stream: bool = True, mmap: bool = False):
    """Read a file written by ``save_mtc``: an MTCMatrix, or a dict name ->
    MTCMatrix for a bundle.

    With ``device`` the matrices' device streams are created there: uploaded
    from the file when it holds a stream of the library's device format
    version (and ``use_stream``), else rebuilt from the host layout."""
    header = read_header(path)
    size = os.path.getsize(path)
    out = {}
    for name, meta in header["entries"].items():
        a = _read_arrays(path, meta["arrays"], mmap, size)
        host = {k: v for k, v in a.items() if not k.startswith(("stream.", "strip."))}
        mat = _build_matrix(name, meta, host)
        pm = meta.get("strip")
        if use_stream and pm is not None:
            from . import strip as _strip

            parrs = {k[len("strip."):]: v for k, v in a.items() if k.startswith("strip.")}
            hs = _strip.import_host(mat, pm, parrs)
            if hs is not None:
                mat.attach_host_strip(hs)
        if device is not None:
            from ..kernels.device import DeviceStream, stream_compatible

            sm = meta.get("stream")
            if use_stream and sm is not None and stream_compatible(sm, mat):
                sarrs = {k[len("stream."):]: v for k, v in a.items() if k.startswith("stream.")}
                mat.attach_device_stream(DeviceStream.from_buffers(mat, device, sm, sarrs))
            else:
                mat.device_stream(device)
        out[name] = mat
    if header.get("single"):
        return out[_SINGLE]
    return out
