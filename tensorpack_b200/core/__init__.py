"""Host-side data model of a packed MTC matrix (reference layout)."""
from .types import PrecisionMode, QRANGE, MODES
from .arena import MemoryArena

__all__ = ["PrecisionMode", "QRANGE", "MODES", "MemoryArena"]
