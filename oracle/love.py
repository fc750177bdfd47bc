"""Float64 restatement of the reference's prediction path.

  alpha solve   kernels/jit/jit_prediction.mojo:681-759 (CG, relative stop)
  LOVE root     jit_prediction.mojo:974-1177 (Lanczos from a hashed +-1 start
                vector, two modified Gram-Schmidt passes, eigenvalue clamp at
                1e-6 lambda_max, S = Q T^{-1/2})
  predictions   jit_prediction.mojo:211-232, 833-870, 1236-1344, 2048-2051
"""
from __future__ import annotations

import math

import numpy as np

from . import kernels as ok

M64 = (1 << 64) - 1


def alpha_cg(A: np.ndarray, b: np.ndarray, max_iter: int, tol: float):
    x = np.zeros_like(b)
    r = b.copy()
    p = b.copy()
    rr_old = float(r @ r)
    r0 = math.sqrt(rr_old) or 1.0
    it = 0
    while it < max_iter:
        Ap = A @ p
        pAp = float(p @ Ap)
        if not (pAp >= 1e-10):
            break
        alpha = rr_old / pAp
        x += alpha * p
        r -= alpha * Ap
        rr_new = float(r @ r)
        it += 1
        if math.sqrt(rr_new) / r0 < tol:
            break
        beta = rr_new / (rr_old + 1e-20) if rr_old >= 1e-20 else 0.0
        beta = 0.0 if (beta < 0 or beta != beta) else beta
        p = r + beta * p
        rr_old = rr_new
    return x, it


def start_vector(n: int, r: int) -> np.ndarray:
    z = np.empty(n)
    for i in range(n):
        s = 0xC0FFEE1234567890 ^ ((i * 0x9E3779B97F4A7C15) & M64) ^ ((r * 0xBF58476D1CE4E5B9) & M64)
        s ^= s >> 12
        s ^= (s << 25) & M64
        s ^= s >> 27
        s = (s * 0x2545F4914F6CDD1D) & M64
        z[i] = 1.0 if (s & 0x20000) else -1.0
    return z / np.linalg.norm(z)


def love_root(A: np.ndarray, r: int) -> np.ndarray:
    """S [n, r] with S S^T ~ A^{-1}."""
    n = A.shape[0]
    Q = np.zeros((r, n))
    alpha = np.zeros(r)
    beta = np.zeros(max(r - 1, 0))
    v = start_vector(n, r)
    Q[0] = v
    v_prev = np.zeros(n)
    beta_prev = 0.0
    for j in range(r):
        w = A @ v
        alpha[j] = v @ w
        w = w - alpha[j] * v
        if j > 0:
            w = w - beta_prev * v_prev
        for _ in range(2):
            max_inner = 0.0
            for k in range(j + 1):
                inner = Q[k] @ w
                max_inner = max(max_inner, abs(inner))
                w = w - inner * Q[k]
            if max_inner < 1e-5:
                break
        bj = np.linalg.norm(w)
        if j < r - 1:
            beta[j] = bj
        if bj < 1e-10:
            Q[j + 1:] = 0.0
            break
        v_prev, v = v, w / bj
        if j + 1 < r:
            Q[j + 1] = v
        beta_prev = bj
    T = np.diag(alpha) + np.diag(beta, 1) + np.diag(beta, -1)
    lam, V = np.linalg.eigh(T)
    lam = np.maximum(lam, max(lam.max(), 1e-10) * 1e-6)
    Tis = (V / np.sqrt(lam)) @ V.T
    return Q.T @ Tis


def predict(spec, params, X, y, noise, mean, Xs, rank, max_cg=300, tol=1e-3):
    X = np.asarray(X, np.float64)
    Xs = np.asarray(Xs, np.float64)
    n = X.shape[0]
    A = ok.kernel_matrix(spec, params, X) + noise * np.eye(n)
    alpha, _ = alpha_cg(A, np.asarray(y, np.float64) - mean, max_cg, tol)
    Ks = ok.kernel_matrix(spec, params, Xs, X)
    mu = Ks @ alpha + mean
    S = love_root(A, rank)
    kss = np.diag(ok.kernel_matrix(spec, params, Xs))
    var = np.maximum(kss - np.sum((Ks @ S) ** 2, axis=1), 1e-10) + noise
    return mu, var, alpha, S
