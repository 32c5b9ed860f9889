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


def linear_fp32_weight(in_features, out_features, seed=42):
    """Weights of the reference's LinearFP32 (mtc/nn/layers.py:78-83):
    uniform(-1/sqrt(in), 1/sqrt(in)) from RandomState(seed)."""
    rng = np.random.RandomState(seed)
    std = 1.0 / np.sqrt(in_features)
    return rng.uniform(-std, std, size=(in_features, out_features)).astype(np.float32)


def heavy_tailed(K, N, seed=9):
    """Student-t(2) weights with a few very large entries (reaches P8/P16)."""
    rng = np.random.default_rng(seed)
    W = rng.standard_t(2, (K, N)).astype(np.float32)
    W[rng.random((K, N)) < 0.002] *= 1e4
    return W


def forced_mode_allocation(K, N, seed=0, sizes=(32, 16, 8, 4), p_split=0.6):
    """Random quadtree tiling whose leaves draw their mode uniformly from all
    eight precisions (P0..P16) at every level, with signed bf16 scales of
    amax/qmax times U(0.6, 1).  The reference allocator never produces this
    mix on its benchmark inputs, so it is the coverage fixture for every
    (edge, mode) pair.  Returns (W, sizes, leaf, modes, scales) with the
    QTAllocation field layout (mtc/core/quadtree.py:55-61)."""
    rng = np.random.default_rng(seed)
    sig = np.exp(rng.uniform(np.log(1e-2), np.log(1e1), (K // 32, N // 32)))
    W = (rng.standard_normal((K, N)) * np.kron(sig, np.ones((32, 32)))).astype(np.float32)
    modes_all = np.array([0, 2, 3, 4, 5, 6, 8, 16], dtype=np.uint8)
    leaf = {s: np.zeros((K // s, N // s), bool) for s in sizes}
    modes = {s: np.zeros((K // s, N // s), np.uint8) for s in sizes}
    scales = {s: np.zeros((K // s, N // s), np.float32) for s in sizes}

    def visit(level, i, j):
        s = sizes[level]
        if level + 1 < len(sizes) and rng.random() < p_split:
            for di in (0, 1):
                for dj in (0, 1):
                    visit(level + 1, 2 * i + di, 2 * j + dj)
            return
        m = int(modes_all[rng.integers(0, 8)])
        leaf[s][i, j] = True
        modes[s][i, j] = m
        if m:
            amax = float(np.abs(W[i * s:(i + 1) * s, j * s:(j + 1) * s]).max())
            qmax = float(2 ** (m - 1) - 1) if m > 2 else 1.0
            sc = np.float32(amax / qmax * rng.uniform(0.6, 1.0) * rng.choice([-1.0, 1.0]))
            scales[s][i, j] = (np.array([sc], np.float32).view(np.uint32) & 0xFFFF0000).view(np.float32)[0]

    root = sizes[0]
    for i in range(K // root):
        for j in range(N // root):
            visit(0, i, j)
    return W, tuple(sizes), leaf, modes, scales


def gptq_layer(K=256, N=256, T=1024, seed=0):
    """A layer with correlated, unevenly scaled input channels and its
    calibration activations (the shape of the GPTQ tests' layer,
    tests/test_gptq.py:13-18): W ~ N(0, 0.05^2), X = N(0,1) @ (I + G/sqrt(K))
    with per-channel log-normal scales."""
    rng = np.random.default_rng(seed)
    W = (rng.standard_normal((K, N)) * 0.05).astype(np.float32)
    mix = rng.standard_normal((K, K)) / np.sqrt(K) + np.eye(K)
    X = (rng.standard_normal((T, K)) @ mix * np.exp(rng.standard_normal(K) * 0.5)).astype(np.float32)
    return W, X
