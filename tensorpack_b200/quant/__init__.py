"""GPU rate-distortion allocators producing MTC-QT / MTC-QT-P allocations,
and the exact reconstructions of those allocations (GPU dequant kernel)."""
from .rd import (Allocation, PermutedAllocation, PermutedQuadtreeRD, QuadtreeRD, channel_orders, index_bits,
                 permuted_qt_dequant, qt_allocate, qt_dequant, unpermute)

__all__ = ["QuadtreeRD", "PermutedQuadtreeRD", "qt_allocate", "Allocation", "PermutedAllocation", "qt_dequant",
           "permuted_qt_dequant", "unpermute", "index_bits", "channel_orders"]
