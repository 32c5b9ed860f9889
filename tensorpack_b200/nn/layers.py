"""Quantized linear layer running the packed MTC GEMM on the GPU.

Drop-in for ``mtc.nn.layers.LinearMTCAdaptive`` (mtc/nn/layers.py:115-151):
same constructor signature, the same seeded fp32 weights (LinearFP32,
layers.py:78-85) packed with ``MTCMatrix.from_numpy`` and the same
``weight_bytes``.  The reference's forward multiplies by a cached dequantised
copy on the CPU; here ``forward`` runs the packed GEMM kernels, so the
packed bytes are what the GPU reads.
"""

from __future__ import annotations

from typing import Optional

import numpy as np
import torch

from ..core.arena import MemoryArena
from ..kernels.gemm import MTCMatrix, gemm_fused, mtc_gemm

_NP_ACT = {
    None: lambda y: y,
    "relu": lambda y: np.where(y < 0, np.float32(0), y),
    "silu": lambda y: y / (np.float32(1) + np.exp(-y)),
    "gelu_tanh": lambda y: np.float32(0.5) * y * (np.float32(1) + np.tanh(
        np.float32(0.7978845608028654) * (y + np.float32(0.044715) * y * y * y))),
}


class LinearFP32:
    """The reference's full-precision linear layer (mtc/nn/layers.py:67-85),
    inference part: seeded uniform(-1/sqrt(in), 1/sqrt(in)) weights,
    ``forward(X) = X @ W + b``.  Kept so that callers which compare the
    quantized layer against it run unchanged; it is not a packed path (numpy
    in, numpy out, as in the reference)."""

    def __init__(self, in_features: int, out_features: int, seed: int = 42):
        rng = np.random.RandomState(seed)
        bound = 1.0 / np.sqrt(in_features)
        self.W = rng.uniform(-bound, bound, size=(in_features, out_features)).astype(np.float32)
        self.b = np.zeros(out_features, dtype=np.float32)

    @property
    def weight_bytes(self) -> int:
        return self.W.nbytes + self.b.nbytes

    def forward(self, X: np.ndarray) -> np.ndarray:
        return np.asarray(X, np.float32) @ self.W + self.b


class LinearMTCAdaptive(torch.nn.Module):
    """``activation`` (None, "relu", "silu", "gelu_tanh") is applied after the
    bias, fused into the GEMM's output pass on the GPU."""

    def __init__(self, in_features: int, out_features: int, block_size: int = 16, epsilon: float = 0.05,
                 seed: int = 42, *, W_mtc: Optional[MTCMatrix] = None, bias: Optional[np.ndarray] = None,
                 activation: Optional[str] = None):
        super().__init__()
        if activation not in _NP_ACT:
            raise ValueError(f"unknown activation {activation!r}")
        self.activation = activation
        self.block_size = block_size
        self.in_features = in_features
        self.out_features = out_features
        if W_mtc is None:
            rng = np.random.RandomState(seed)
            std = 1.0 / np.sqrt(in_features)
            W = rng.uniform(-std, std, size=(in_features, out_features)).astype(np.float32)
            self.arena = MemoryArena(capacity_bytes=in_features * out_features * 2)
            W_mtc = MTCMatrix.from_numpy(W, block_size=block_size, epsilon=epsilon, arena=self.arena,
                                         use_pointer_hierarchy=False)
        else:
            if W_mtc.shape != (in_features, out_features):
                raise ValueError(f"W_mtc shape {W_mtc.shape} != ({in_features}, {out_features})")
            self.arena = W_mtc.arena
        self.W_mtc = W_mtc
        self.b = np.zeros(out_features, dtype=np.float32) if bias is None else np.asarray(bias, np.float32)
        self._bias_dev = {}

    @classmethod
    def from_mtc(cls, W_mtc: MTCMatrix, bias: Optional[np.ndarray] = None,
                 activation: Optional[str] = None) -> "LinearMTCAdaptive":
        """Wrap an already packed matrix (e.g. from ``MTCMatrix.from_qt_allocation``)."""
        K, N = W_mtc.shape
        return cls(K, N, block_size=W_mtc.block_size, W_mtc=W_mtc, bias=bias, activation=activation)

    @property
    def weight_bytes(self) -> int:
        return self.W_mtc.total_bytes_allocated + self.b.nbytes

    def forward(self, X):
        if isinstance(X, np.ndarray):
            return _NP_ACT[self.activation](mtc_gemm(X, self.W_mtc) + self.b)
        if X.device.type != "cuda":
            raise ValueError("LinearMTCAdaptive: activations must be a CUDA tensor (no CPU path)")
        key = str(X.device)
        bd = self._bias_dev.get(key)
        if bd is None:
            bd = torch.from_numpy(self.b).to(X.device)
            self._bias_dev[key] = bd
        return gemm_fused(X, self.W_mtc, bd, self.activation)


def fold_layers(a: LinearMTCAdaptive, b: LinearMTCAdaptive):
    """(a', b') computing b(a(X)) with a's output left in its stored column
    order and b's input permutation absorbing it (tensorpack_b200.kernels.
    fold): no column scatter after a, and a' outputs act(Y_a)[:, pc_a]."""
    from ..kernels.fold import fold_permutation

    wa, wb = fold_permutation(a.W_mtc, b.W_mtc)
    pc = a.W_mtc.col_perm
    bias_a = a.b if pc is None else a.b[np.asarray(pc)]
    return (LinearMTCAdaptive.from_mtc(wa, bias_a, a.activation), LinearMTCAdaptive.from_mtc(wb, b.b, b.activation))
