"""Seeded synthetic inputs shared by the fixture generator, the tests and the bench.

Each generator reproduces the shape and value distribution of one of the
reference's test or benchmark inputs (cited per function); the values come
from numpy's default generator so every machine with the same numpy rebuilds
the same matrices.
"""

import numpy as np


def outlier_matrix(n=128, seed=0):
    """Small Gaussian weights with 1 % large outliers (the shape used by the
    quadtree tests, tests/test_quadtree.py:14-19)."""
    rng = np.random.default_rng(seed)
    W = (rng.standard_normal((n, n)) * 0.05).astype(np.float32)
    mask = rng.random((n, n)) < 0.01
    W[mask] = rng.uniform(-25, 25, size=int(mask.sum())).astype(np.float32)
    return W


def row_scaled(K=256, N=256, seed=0):
    """Rows of log-normally varying scale in random order plus a positive
    importance vector (tests/test_permutation.py:15-20)."""
    rng = np.random.default_rng(seed)
    W = (rng.standard_normal((K, N)) * np.exp(rng.standard_normal((K, 1)))).astype(np.float32)
    h = np.exp(rng.standard_normal(K) * 0.5)
    return W, h


def llm_like(K, N, seed=0, calib_rows=512):
    """Student-t(4) * 0.02 weights and the mean-square importance of
    calibration activations whose 1 % outlier channels are scaled x50
    (mtc/benchmarks/benchmark_pareto.py:141-153 and BASELINE.json configs)."""
    rng = np.random.default_rng(seed)
    W = (rng.standard_t(4, (K, N)) * 0.02).astype(np.float32)
    sc = np.ones(K, np.float32)
    sc[rng.choice(K, max(K // 100, 1), replace=False)] = 50.0
    Xc = (rng.standard_normal((calib_rows, K)) * sc).astype(np.float32)
    h = (Xc.astype(np.float64) ** 2).mean(axis=0)
    return W, h


def llm_activations(M, K, seed=0, outlier_seed=None):
    """Activations with the same 1 %-outlier channel structure (x50)."""
    rng = np.random.default_rng(seed)
    sc = np.ones(K, np.float32)
    orng = np.random.default_rng(seed if outlier_seed is None else outlier_seed)
    sc[orng.choice(K, max(K // 100, 1), replace=False)] = 50.0
    return (rng.standard_normal((M, K)) * sc).astype(np.float32)


def multiscale(n=256, seed=2):
    """Each 32x32 block N(0, sigma^2), sigma^2 log-uniform on [1e-3, 1e2]
    (BASELINE.json multi-scale stress config)."""
    rng = np.random.default_rng(seed)
    var = np.exp(rng.uniform(np.log(1e-3), np.log(1e2), (n // 32, n // 32)))
    sig = np.kron(np.sqrt(var), np.ones((32, 32)))
    return (rng.standard_normal((n, n)) * sig).astype(np.float32)


def cpu_ref_config():
    """W 1024x1024 ~N(0,1), X_cal 256x1024 ~N(0,1),
    h = mean(X_cal^2), X 256x1024 ~N(0,1), seed 0."""
    rng = np.random.default_rng(0)
    W = rng.standard_normal((1024, 1024)).astype(np.float32)
    Xc = rng.standard_normal((256, 1024)).astype(np.float32)
    h = (Xc.astype(np.float64) ** 2).mean(axis=0)
    X = rng.standard_normal((256, 1024)).astype(np.float32)
    return W, h, X


def fixed_pair(seed=5):
    """A 128x96 with silent columns, B 96x64 with a loud row band
    (tests/test_allocation.py:69-76)."""
    rng = np.random.default_rng(seed)
    A = rng.standard_normal((128, 96)).astype(np.float32)
    B = rng.standard_normal((96, 64)).astype(np.float32)
    A[:, :32] *= 1e-4
    B[32:64] *= 20.0
    return A, B
