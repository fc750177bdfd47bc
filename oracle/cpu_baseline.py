"""CPU baseline for the matvec metric — the reference's CPU route, restated.

The reference's CPU path for a kernel matrix is its NumPy evaluator
(mojogp/kernel.py:804-923): scale inputs by the lengthscales, form squared
distances by the expansion |x|^2 + |y|^2 - 2 x.y with a BLAS matmul, clamp at
0, exponentiate, scale by the outputscale. The matrix-free product K V is that
evaluator applied block by block (row block x all columns) followed by a BLAS
K_block @ V, in float64 as the evaluator computes. Row blocks are spread over
host threads (NumPy releases the GIL inside BLAS and ufuncs).

Used only by bench.py (cpu_baseline field and the --impl reference arm); the
product never calls it.
"""
from __future__ import annotations

import os
import time
from concurrent.futures import ThreadPoolExecutor

import numpy as np


def rbf_ard_block(Xr: np.ndarray, Xc: np.ndarray, ell: np.ndarray, os_: float) -> np.ndarray:
    """K(Xr, Xc) for RBF-ARD following kernel.py:876-900 (float64)."""
    A = Xr / ell
    B = Xc / ell
    sq = (A * A).sum(1)[:, None] + (B * B).sum(1)[None, :] - 2.0 * (A @ B.T)
    np.maximum(sq, 0.0, out=sq)
    return os_ * np.exp(-0.5 * sq)


def matvec_rows(X: np.ndarray, V: np.ndarray, ell: np.ndarray, os_: float, rows: np.ndarray,
                row_block: int = 64, col_block: int = 16384, threads: int | None = None) -> np.ndarray:
    """(K V)[rows] by blocks; returns [len(rows), t] float64."""
    X64 = X.astype(np.float64, copy=False)
    V64 = V.astype(np.float64, copy=False)
    ell = np.asarray(ell, np.float64)
    out = np.zeros((len(rows), V.shape[1]))
    chunks = [rows[i:i + row_block] for i in range(0, len(rows), row_block)]

    def work(ci):
        r = chunks[ci]
        acc = np.zeros((len(r), V.shape[1]))
        Xr = X64[r]
        for c0 in range(0, X.shape[0], col_block):
            acc += rbf_ard_block(Xr, X64[c0:c0 + col_block], ell, os_) @ V64[c0:c0 + col_block]
        return ci, acc

    threads = threads or (os.cpu_count() or 1)
    with ThreadPoolExecutor(max_workers=threads) as ex:
        for ci, acc in ex.map(work, range(len(chunks))):
            out[ci * row_block: ci * row_block + len(chunks[ci])] = acc
    return out


def time_matvec_sample(X, V, ell, os_, target_s: float = 15.0, threads: int | None = None,
                       max_rows: int = 4096):
    """Time the CPU route on a bounded row sample; returns dict with pairs/s."""
    threads = threads or (os.cpu_count() or 1)
    n = X.shape[0]
    rows = np.arange(min(64, n))
    t0 = time.perf_counter()
    matvec_rows(X, V, ell, os_, rows, threads=threads)
    dt = time.perf_counter() - t0
    nrows = int(min(max_rows, n, max(64, 64 * target_s / max(dt, 1e-3) * min(threads, 8) / 2)))
    nrows = max(64, nrows // 64 * 64)
    rows = np.arange(nrows)
    t0 = time.perf_counter()
    matvec_rows(X, V, ell, os_, rows, threads=threads)
    dt = time.perf_counter() - t0
    pairs = nrows * n
    return {"seconds": dt, "rows": nrows, "pairs": pairs, "pairs_per_s": pairs / dt,
            "threads": threads}


def exact_fit_iteration(X, y, ell, os_, noise):
    """One fit iteration of the reference's NumPy exact-Cholesky route
    (tests/integration/test_exactgp_variance_accuracy.py:30-46 and
    tests/shared/dense_references.py:67-82 restated): RBF kernel matrix,
    Cholesky of K + noise I, alpha, the log marginal likelihood per sample and
    its gradient w.r.t. (lengthscales, outputscale, noise) through
    0.5 tr((alpha alpha^T - K^-1) dK). Returns (nll, gradient)."""
    Xs = np.asarray(X, np.float64) / np.asarray(ell, np.float64)
    n = Xs.shape[0]
    sq = (Xs * Xs).sum(1)
    D = np.maximum(sq[:, None] + sq[None, :] - 2.0 * Xs @ Xs.T, 0.0)
    E = np.exp(-0.5 * D)
    K = os_ * E
    Ky = K + noise * np.eye(n)
    L = np.linalg.cholesky(Ky)
    alpha = np.linalg.solve(L.T, np.linalg.solve(L, np.asarray(y, np.float64)))
    Kinv = np.linalg.solve(L.T, np.linalg.solve(L, np.eye(n)))
    W = np.outer(alpha, alpha) - Kinv
    nll = (0.5 * y @ alpha + np.log(np.diag(L)).sum() + 0.5 * n * np.log(2 * np.pi)) / n
    grads = []
    for k in range(Xs.shape[1]):
        dk = Xs[:, k][:, None] - Xs[:, k][None, :]
        grads.append(-0.5 * (W * (K * dk * dk / ell[k])).sum() / n)
    grads.append(-0.5 * (W * E).sum() / n)
    grads.append(-0.5 * np.trace(W) / n)
    return float(nll), np.array(grads)


def time_exact_fit_iteration(X, y, ell, os_, noise, reps: int = 3):
    """Median seconds of exact_fit_iteration over `reps` runs (BLAS threads as set)."""
    ts = []
    for _ in range(reps):
        t0 = time.perf_counter()
        exact_fit_iteration(X, y, ell, os_, noise)
        ts.append(time.perf_counter() - t0)
    return float(np.median(ts))
