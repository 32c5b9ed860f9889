"""GPU rate-distortion allocators producing MTC-QT / MTC-QT-P allocations."""
from .rd import PermutedQuadtreeRD, QuadtreeRD

__all__ = ["QuadtreeRD", "PermutedQuadtreeRD"]
