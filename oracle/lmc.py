"""Float64 restatement of the LMC (linear model of coregionalisation) BBMM.

  operator   K_full = sum_s A_s (x) K_s + diag(noise_t) (x) I_n, task-blocked
             (kernels/jit/jit_lmc.mojo:275-330, lmc_provider.mojo:113-192)
  gradients  kernel params through A_s (x) dK_s; A_s and per-task noise
             (jit_lmc.mojo:582-691); NLL / SLQ as combined_inv_quad_logdet.mojo:452
  precond    sum-of-Kronecker Woodbury P = sum_s A_s (x) L_s L_s^T + D
             (lmc_preconditioner.mojo:143-470, built as jit_lmc.mojo:848-900);
             probes use the library's counter-hash Gaussians (omega seed s,
             eps seed s + 1e6) instead of the reference's host generator, so
             preconditioned runs are pinned to this restatement, not to the
             reference's random stream.
Test infrastructure only (tests, smoke checks, CPU baseline).
"""
from __future__ import annotations

import math

import numpy as np

from . import bbmm as ob
from . import kernels as ok


def full_operator(specs, params_list, X, A, noise):
    n = X.shape[0]
    T = A.shape[1]
    Ks, Gs = [], []
    K = np.kron(np.diag(noise), np.eye(n))
    for s, (spec, p) in enumerate(zip(specs, params_list)):
        Kx, G = ok.kernel_matrix(spec, p, X, want_grad=True)
        Ks.append(Kx)
        Gs.append(G)
        K = K + np.kron(A[s], Kx)
    return K, Ks, Gs


def exact_variance(specs, params_list, X, Xtest, A, noise):
    """Exact LMC posterior variance [m, T] (_predict_lmc_full_exact_variance_backend,
    mojogp/multi_output_gp.py:4360-4519): for test point c and task t,
    max(sum_s A_s[t, t] k_s(x*, x*) - r^T K_full^{-1} r + noise_t, 1e-10) with
    r = sum_s A_s[:, t] (x) k_s(X, x*_c), by a dense float64 solve."""
    K, _, _ = full_operator(specs, params_list, X, A, noise)
    m, T = Xtest.shape[0], A.shape[1]
    R = len(specs)
    prior = np.zeros((m, T))
    Rhs = np.zeros((K.shape[0], m * T))
    for s, (spec, p) in enumerate(zip(specs, params_list)):
        Kc = ok.kernel_matrix(spec, p, X, Xtest)  # [n, m]
        kd = np.array([ok.kernel_matrix(spec, p, Xtest[c:c + 1])[0, 0] for c in range(m)])
        prior += kd[:, None] * np.diag(A[s])[None, :]
        for t in range(T):
            Rhs[:, t::T] += np.kron(A[s][:, t:t + 1], Kc)
    Sol = np.linalg.solve(K, Rhs)
    corr = np.einsum("ij,ij->j", Rhs, Sol).reshape(m, T)
    return np.maximum(prior - corr + np.asarray(noise)[None, :], 1e-10)


class LmcPrecond:
    """P = sum_s (C_s (x) L_s)(C_s (x) L_s)^T + D; Woodbury apply, log|P|, N(0, P) probes."""

    def __init__(self, Ks, A, noise, rank, factor_dtype=np.float64):
        A = np.asarray(A, np.float64)
        self.R, self.T = A.shape[0], A.shape[1]
        self.n = Ks[0].shape[0]
        self.noise = np.asarray(noise, np.float64)
        # greedy pivoted Cholesky of each K_s
        self.L = [ob.Precond(K, 1.0, rank, factor_dtype).L for K in Ks]
        self.C = []
        for s in range(self.R):
            try:
                self.C.append(np.linalg.cholesky(A[s]))
            except np.linalg.LinAlgError:
                self.C.append(np.linalg.cholesky(A[s] + 1e-4 * np.eye(self.T)))
        # U = [C_s (x) L_s] with column order (s, j, k) -> off_s + j r_s + k
        self.U = np.concatenate([np.kron(self.C[s], self.L[s]) for s in range(self.R)], axis=1)
        self.d = np.repeat(self.noise, self.n)
        M = np.eye(self.U.shape[1]) + self.U.T @ (self.U / self.d[:, None])
        self.Minv = np.linalg.inv(M)
        _, ldM = np.linalg.slogdet(M)
        self.logdet = self.n * float(np.sum(np.log(self.noise))) + ldM
        self.ranks = [L.shape[1] for L in self.L]

    def dense(self):
        return self.U @ self.U.T + np.diag(self.d)

    def apply(self, V):
        w = V / self.d[:, None]
        return w - (self.U @ (self.Minv @ (self.U.T @ w))) / self.d[:, None]

    def sample(self, num, seed):
        nT = self.n * self.T
        Kt = self.U.shape[1]
        eps = ob.gaussian_block(nT, num, seed + 1000000)
        om = ob.hash_gaussian(np.arange(num * Kt, dtype=np.uint64), seed).reshape(num, Kt).T
        return np.sqrt(self.d)[:, None] * eps + self.U @ om


def lmc_bbmm(specs, params_list, X, Y_centered, A, noise, num_probes, max_cg, max_tridiag, tol,
             iteration=0, precond_rank=0, precond=None, x_prev=None):
    """Y_centered [n, T]. Returns nll, kernel grads (concatenated), grad_A, grad_noise.
    `precond` (an LmcPrecond) is used as given, e.g. one built at an earlier
    state; else precond_rank > 0 builds one here. `x_prev` starts the data
    column's CG from a previous normalised solution (recycle_alpha,
    combined_inv_quad_logdet.mojo); the result's x_norm0 is this solve's."""
    X = np.asarray(X, np.float64)
    n = X.shape[0]
    A = np.asarray(A, np.float64)
    T = A.shape[1]
    nT = n * T
    y = np.asarray(Y_centered, np.float64).T.reshape(nT)  # task-blocked
    K, Ks, Gs = full_operator(specs, params_list, X, A, np.asarray(noise, np.float64))
    seed = iteration * 104729 + 42
    P = precond if precond is not None else \
        (LmcPrecond(Ks, A, noise, precond_rank) if precond_rank > 0 else None)
    Z = P.sample(num_probes, seed) if P is not None else ob.gaussian_block(nT, num_probes, seed)
    pn = np.linalg.norm(Z, axis=0)
    rhs = np.concatenate([y[:, None], Z / pn], axis=1)
    rn = np.linalg.norm(rhs, axis=0)
    x0 = None
    if x_prev is not None:
        x0 = np.zeros_like(rhs)
        x0[:, 0] = x_prev
    x, iters, dg, od = ob.mbcg(K, rhs / rn, max_cg, max_tridiag, tol, P, x0)
    W = P.apply(Z) if P is not None else Z  # right factors
    sol = x * rn
    alpha = sol[:, 0]
    U = sol[:, 1:] * pn
    inv_quad = float(y @ alpha)
    logdet = ob.slq_logdet(dg[1:], od[1:], nT) + (P.logdet if P is not None else 0.0)
    PI = float(np.float32(3.14159265358979323846))
    nll = (0.5 * inv_quad + 0.5 * logdet + 0.5 * nT * math.log(2 * PI)) / nT
    kgrads = []
    for s in range(len(Ks)):
        for g in Gs[s]:
            dK = np.kron(A[s], g)
            kgrads.append((-0.5 * alpha @ dK @ alpha + 0.5 * np.sum(U * (dK @ W)) / num_probes) / nT)
    blk = lambda v, t: v[t * n:(t + 1) * n]
    gA = np.zeros_like(A)
    for s in range(len(Ks)):
        for i in range(T):
            for j in range(T):
                d = blk(alpha, i) @ Ks[s] @ blk(alpha, j)
                tr = sum(blk(U[:, k], i) @ Ks[s] @ blk(W[:, k], j) for k in range(num_probes))
                gA[s, i, j] = 0.5 * (-d + tr / num_probes) / nT
    gn = np.array([0.5 * (-blk(alpha, t) @ blk(alpha, t)
                          + sum(blk(U[:, k], t) @ blk(W[:, k], t) for k in range(num_probes))
                          / num_probes) / nT for t in range(T)])
    sum_alpha = np.array([blk(alpha, t).sum() for t in range(T)])
    return {"nll": nll, "kgrads": np.array(kgrads), "gA": gA, "gnoise": gn,
            "sum_alpha": sum_alpha, "cg_iters": iters, "K": K, "Ks": Ks, "alpha": alpha,
            "x_norm0": x[:, 0]}
