"""Precision modes of MTC micro-tensors (mtc/core/types.py:9-28) and their
signed code ranges (mtc/core/allocation.py:44-52)."""

from enum import IntEnum
from typing import Dict, Tuple


class PrecisionMode(IntEnum):
    """Bits per code; P0 is a dropped block (all zeros, no payload)."""

    P0 = 0
    P2 = 2
    P3 = 3
    P4 = 4
    P5 = 5
    P6 = 6
    P8 = 8
    P16 = 16

    @property
    def values_per_byte(self) -> float:
        return float("inf") if self.value == 0 else 8.0 / self.value

    @property
    def bytes_per_value(self) -> float:
        return self.value / 8.0


# Signed code range per mode.
QRANGE: Dict[int, Tuple[int, int]] = {
    2: (-2, 1), 3: (-4, 3), 4: (-8, 7), 5: (-16, 15), 6: (-32, 31), 8: (-128, 127), 16: (-32768, 32767),
}
MODES = (0, 2, 3, 4, 5, 6, 8, 16)
# Stored metadata per leaf for each scale format: scale + one mode byte
# (mtc/core/allocation.py:197).
META_BITS = {"fp32": 40, "bf16": 24}
# One split flag per quadtree node above the finest level (mtc/core/quadtree.py:40).
SPLIT_FLAG_BITS = 1
