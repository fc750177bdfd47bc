"""Seeded synthetic workloads for the five benchmark configurations.

No dataset is named by the benchmark; these generators follow the recipes of
the configuration list (draws taken from numpy.random.default_rng(seed) in the
order written). They are used by bench.py, the tests and the examples.
"""
from __future__ import annotations

import numpy as np


def config1(seed: int = 0):
    """n=2000 1-D: X = linspace(-3, 3), y = sin(2x) + 0.05 N(0,1); X* = linspace(-4, 4, 128)."""
    rng = np.random.default_rng(seed)
    X = np.linspace(-3, 3, 2000, dtype=np.float32)[:, None]
    y = (np.sin(2 * X[:, 0]) + 0.05 * rng.standard_normal(2000)).astype(np.float32)
    Xs = np.linspace(-4, 4, 128, dtype=np.float32)[:, None]
    return X, y, Xs


def config2(seed: int = 2, n: int = 100_000, d: int = 8):
    """X ~ U[0,1]^d, w ~ U[0.5, 2]^d, y = sum_k sin(2 pi x_k w_k) + 0.1 N(0,1)."""
    rng = np.random.default_rng(seed)
    X = rng.uniform(0, 1, size=(n, d)).astype(np.float32)
    w = rng.uniform(0.5, 2.0, size=d)
    y = (np.sin(2 * np.pi * X * w).sum(axis=1) + 0.1 * rng.standard_normal(n)).astype(np.float32)
    return X, y


def config3(seed: int = 3, n: int = 1_000_000, d: int = 16, features: int = 256):
    """X ~ N(0, I), l ~ U[0.5, 3]^d, y = RFF GP-prior draw + 0.05 N(0,1).

    Returns X, y, lengthscales.
    """
    rng = np.random.default_rng(seed)
    X = rng.standard_normal((n, d)).astype(np.float32)
    ell = rng.uniform(0.5, 3.0, size=d)
    omega = rng.standard_normal((features, d))
    b = rng.uniform(0, 2 * np.pi, size=features)
    a = rng.standard_normal(features)
    f = np.empty(n, dtype=np.float64)
    blk = 65536
    for i in range(0, n, blk):
        Z = (X[i:i + blk] / ell) @ omega.T + b
        f[i:i + blk] = np.sqrt(2.0 / features) * (np.cos(Z) @ a)
    y = (f + 0.05 * rng.standard_normal(n)).astype(np.float32)
    return X, y, ell.astype(np.float32)


def config4(seed: int = 4, n: int = 50_000, d: int = 4, T: int = 4, features: int = 256):
    """LMC: 3 latent RFF draws (RBF l=0.5; Matern-3/2 l=0.5; RBF-ARD l~U[0.3,1]^d),
    W ~ N(0,1)^{T x 3}, Y = latents W^T + 0.05 N(0,1). Returns X, Y."""
    rng = np.random.default_rng(seed)
    X = rng.uniform(-1, 1, size=(n, d)).astype(np.float32)

    def rff(omega, ell):
        b = rng.uniform(0, 2 * np.pi, size=features)
        a = rng.standard_normal(features)
        Z = (X / ell) @ omega.T + b
        return np.sqrt(2.0 / features) * (np.cos(Z) @ a)

    l1 = rff(rng.standard_normal((features, d)), 0.5)
    # Matern-3/2 spectral density: multivariate Student-t with 3 dof.
    g = rng.standard_normal((features, d))
    chi = rng.chisquare(3, size=(features, 1))
    l2 = rff(g / np.sqrt(chi / 3.0), 0.5)
    ell3 = rng.uniform(0.3, 1.0, size=d)
    l3 = rff(rng.standard_normal((features, d)), ell3)
    W = rng.standard_normal((T, 3))
    lat = np.stack([l1, l2, l3], axis=1)
    Y = (lat @ W.T + 0.05 * rng.standard_normal((n, T))).astype(np.float32)
    return X, Y


def config5(seed: int = 5, n: int = 1_000_000, n_test: int = 1_000_000, d: int = 8):
    """LOVE at scale: X, X* ~ U[0,1]^d, fixed RBF-ARD hyperparameters
    l ~ U[0.2, 1], os = 1, noise = 0.01. Returns X, y, X*, params, noise."""
    rng = np.random.default_rng(seed)
    X = rng.uniform(0, 1, size=(n, d)).astype(np.float32)
    Xs = rng.uniform(0, 1, size=(n_test, d)).astype(np.float32)
    ell = rng.uniform(0.2, 1.0, size=d).astype(np.float32)
    y = (np.sin(2 * np.pi * X[:, 0]) + 0.1 * rng.standard_normal(n)).astype(np.float32)
    params = np.concatenate([ell, [1.0]]).astype(np.float32)
    return X, y, Xs, params, 0.01


def probes_v(n: int, t: int, seed: int = 0) -> np.ndarray:
    """Column block [n, t] of standard normals for isolated matvec runs."""
    return np.random.default_rng(seed).standard_normal((n, t)).astype(np.float32)
