"""Loading saved matrices onto the GPU (tensorpack_b200.core.fileformat).

A file saved with its device stream is uploaded without the repack; the
uploaded stream must equal a fresh repack byte for byte, dequantise
bit-exactly to the oracle and give bit-identical GEMM results.  A file whose
stream was made by another device format version is repacked instead.
"""

import json
import struct

import numpy as np
import pytest

import inputs
from oracle import mtc_oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    import torch

    from tensorpack_b200 import build

    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    build.build()
    return torch.device("cuda", 0)


def _matrix():
    from tensorpack_b200.kernels.gemm import MTCMatrix

    W, sizes, leaf, modes, scales = inputs.forced_mode_allocation(192, 800, seed=13, p_split=0.5)
    rng = np.random.default_rng(3)
    pr, pc = rng.permutation(192), rng.permutation(800)
    inner = O.QuadtreeAllocation(sizes, leaf, modes, scales, None, 0)
    alloc = O.PermutedAllocation(inner, pr, pc, None, 0)
    ref = O.permuted_quadtree_dequant(W, pr, pc, sizes, leaf, modes, scales)
    return MTCMatrix.from_qt_allocation(W, alloc), ref


def _bump_stream_version(path):
    raw = bytearray(open(path, "rb").read())
    magic, ver, hlen, data_off = struct.unpack("<8sIIQ", raw[:24])
    h = json.loads(raw[24:24 + hlen])
    h["entries"]["matrix"]["stream"]["version"] += 100
    blob = json.dumps(h, sort_keys=True).encode()
    assert 24 + len(blob) <= data_off
    raw[12:16] = struct.pack("<I", len(blob))
    raw[24:data_off] = blob + b"\0" * (data_off - 24 - len(blob))
    open(path, "wb").write(bytes(raw))


def test_saved_stream_uploads_and_matches_repack(dev, tmp_path):
    import torch

    from tensorpack_b200.kernels.device import _STREAM_ARRAYS
    from tensorpack_b200.kernels.gemm import MTCMatrix

    m, ref = _matrix()
    ds = m.device_stream(dev)
    p = tmp_path / "m.mtcpk"
    m.save(p, include_stream=True, device=dev)
    r = MTCMatrix.load(p, device=dev)
    rs = r.device_stream(dev)
    assert rs.source == "file" and ds.source == "repack"
    for name in _STREAM_ARRAYS:
        assert torch.equal(getattr(rs, name), getattr(ds, name)), name
    np.testing.assert_array_equal(rs.dequant(original_order=True).cpu().numpy(), ref)
    for M in (1, 7, 300):
        X = torch.from_numpy(inputs.llm_activations(M, 192, seed=M, outlier_seed=1)).to(dev)
        Y0 = torch.empty(M, 800, device=dev)
        Y1 = torch.empty(M, 800, device=dev)
        ds.matmul(X, Y0)
        rs.matmul(X, Y1)
        torch.cuda.synchronize()
        ds.check_status()
        rs.check_status()
        assert torch.equal(Y0, Y1), M


def test_stream_of_another_version_is_repacked(dev, tmp_path):
    from tensorpack_b200.kernels.gemm import MTCMatrix

    m, ref = _matrix()
    p = tmp_path / "old.mtcpk"
    m.save(p, include_stream=True, device=dev)
    _bump_stream_version(p)
    r = MTCMatrix.load(p, device=dev)
    rs = r.device_stream(dev)
    assert rs.source == "repack"
    np.testing.assert_array_equal(rs.dequant(original_order=True).cpu().numpy(), ref)
