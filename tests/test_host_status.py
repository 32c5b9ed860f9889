"""Host handling of the kernels' status word (no GPU needed).

A kernel that gives up part-way (a bounded wait that ran out, a tile record
that failed a bounds check, activations beyond the fp16 range) sets
MTC_STATUS_* bits; ``DeviceStream.check_status`` turns them into a
RuntimeError and restores the zero state of the split-K ticket arrays that
the next call relies on.
"""

import pytest
import torch

from tensorpack_b200 import _lib
from tensorpack_b200.kernels.device import DeviceStream


def stream_with(status):
    ds = DeviceStream.__new__(DeviceStream)
    ds.status = torch.tensor([status], dtype=torch.int32)
    ds.counters = torch.tensor([3, 0, 1], dtype=torch.int32)
    ds.decode_counters = torch.tensor([2, 5, 0, 0, 1, 0], dtype=torch.int32)
    return ds


def test_clean_status_leaves_state_alone():
    ds = stream_with(0)
    ds.check_status()
    assert ds.counters.tolist() == [3, 0, 1]
    assert ds.decode_counters.tolist() == [2, 5, 0, 0, 1, 0]


@pytest.mark.parametrize("bits,text", [
    (_lib.STATUS_TIMEOUT, "timed out"),
    (_lib.STATUS_X_RANGE, "fp16 range"),
    (_lib.STATUS_BAD_STREAM, "bounds check"),
    (_lib.STATUS_TIMEOUT | _lib.STATUS_BAD_STREAM, "timed out; tile stream"),
])
def test_failed_call_raises_and_clears_tickets(bits, text):
    ds = stream_with(bits)
    with pytest.raises(RuntimeError, match=text):
        ds.check_status()
    assert int(ds.status.item()) == 0
    assert not ds.counters.any() and not ds.decode_counters.any()
    ds.check_status()  # reported once
