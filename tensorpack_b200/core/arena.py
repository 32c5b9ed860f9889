"""Contiguous byte arena holding packed payloads (mtc/core/arena.py:9-75).

Same interface as the reference: a growable ``uint8`` buffer with bump
allocation and ``uint32``-sized offsets.  It is the host copy of the
reference layout; the GPU path repacks it into a device tile stream.
"""

import numpy as np


class MemoryArena:
    def __init__(self, capacity_bytes: int = 64 * 1024 * 1024):
        self._capacity = int(capacity_bytes)
        self._buffer = np.zeros(self._capacity, dtype=np.uint8)
        self._offset = 0

    @property
    def capacity(self) -> int:
        return self._capacity

    @property
    def bytes_allocated(self) -> int:
        return self._offset

    @property
    def utilization_pct(self) -> float:
        return (self._offset / self._capacity) * 100.0 if self._capacity > 0 else 0.0

    @property
    def raw_buffer(self) -> np.ndarray:
        return self._buffer

    def allocate(self, size_bytes: int, alignment: int = 1) -> int:
        """Reserve ``size_bytes`` (aligned start), growing x2 when full."""
        if alignment > 1 and self._offset % alignment:
            self._offset += alignment - self._offset % alignment
        start = self._offset
        end = start + int(size_bytes)
        if end > self._capacity:
            cap = max(self._capacity * 2, end + 1024 * 1024)
            buf = np.zeros(cap, dtype=np.uint8)
            buf[:start] = self._buffer[:start]
            self._buffer, self._capacity = buf, cap
        self._offset = end
        return start

    def write_bytes(self, data, alignment: int = 1) -> int:
        flat = np.asarray(data, dtype=np.uint8).ravel()
        off = self.allocate(flat.nbytes, alignment)
        self._buffer[off:off + flat.nbytes] = flat
        return off

    def view(self, offset: int, length: int) -> np.ndarray:
        return self._buffer[offset:offset + length]

    def reset(self):
        self._offset = 0
