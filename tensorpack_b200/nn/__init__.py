"""Quantized linear layer on the packed MTC GEMM (drop-in for mtc.nn)."""
from .layers import LinearMTCAdaptive

__all__ = ["LinearMTCAdaptive"]
