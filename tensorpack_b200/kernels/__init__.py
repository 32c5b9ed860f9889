"""Packed MTC GEMM (drop-in for mtc.kernels.gemm)."""
from .gemm import MTCMatrix, mtc_gemm

__all__ = ["MTCMatrix", "mtc_gemm"]
