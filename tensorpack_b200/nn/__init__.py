"""Quantized linear layer on the packed MTC GEMM (drop-in for mtc.nn), and
the full-precision layer that callers compare it with."""
from .layers import LinearFP32, LinearMTCAdaptive

__all__ = ["LinearMTCAdaptive", "LinearFP32"]
