"""The bounded-wait path of the strip decode, made to run out on purpose.

A diagnostic hold (mtc_debug_withhold_bytes) makes the first batch of every
warp expect 16 bytes that no copy delivers, so that mbarrier phase never
completes: each wait gives up at the (shortened) limit, the call reports
MTC_STATUS_TIMEOUT through the status word, drains its own copies and
returns, and the next call on the same stream is correct.  Nothing here
faults or hangs the GPU: every wait is bounded.
"""

import numpy as np
import pytest

import inputs
from oracle import mtc_oracle as O
from strip_emul import emulated_product

pytestmark = pytest.mark.gpu


def test_strip_wait_runs_out_and_next_call_is_correct():
    import torch

    from tensorpack_b200 import _lib, build
    from tensorpack_b200.kernels.gemm import MTCMatrix

    assert torch.cuda.is_available()
    build.build()
    lib = _lib.load()
    dev = torch.device("cuda", 0)
    W, sizes, leaf, modes, scales = inputs.forced_mode_allocation(256, 384, seed=11, p_split=0.5)
    m = MTCMatrix.from_qt_allocation(W, O.QuadtreeAllocation(sizes, leaf, modes, scales, None, 0))
    deq = O.quadtree_dequant(W, sizes, leaf, modes, scales)
    ds = m.device_stream(dev)
    X = np.random.default_rng(4).standard_normal((2, 256)).astype(np.float32)
    Xd = torch.from_numpy(X).to(dev)
    Y = torch.full((2, 384), float("nan"), device=dev)
    ds.decode_strip(Xd, Y)  # build and upload the strip stream before timing anything
    torch.cuda.synchronize()
    ds.check_status()
    try:
        assert lib.mtc_set_wait_limit_ns(1_000_000) == 0  # 1 ms
        assert lib.mtc_debug_withhold_bytes(16) == 0
        Y.fill_(float("nan"))
        ds.decode_strip(Xd, Y)  # returns at once: the kernel runs asynchronously
        torch.cuda.synchronize()  # the kernel ended: no wait outlived its limit
        st = int(ds.status.item())
        assert st & _lib.STATUS_TIMEOUT, st
        assert torch.isnan(Y).all(), "a CTA that gave up must not write its output"
        with pytest.raises(RuntimeError, match="timed out"):
            ds.check_status()  # raises and clears the status word
        assert int(ds.status.item()) == 0
    finally:
        lib.mtc_debug_withhold_bytes(0)
        lib.mtc_set_wait_limit_ns(0)
    ds.decode_strip(Xd, Y)
    torch.cuda.synchronize()
    ds.check_status()
    emul, _ = emulated_product(m, deq, X, ds.strip().host.exp2)
    assert O.relative_frobenius_error(emul, Y.cpu().numpy()) < 1e-5

