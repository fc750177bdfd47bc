"""Float64 restatement of the LMC (linear model of coregionalisation) BBMM.

  operator   K_full = sum_s A_s (x) K_s + diag(noise_t) (x) I_n, task-blocked
             (kernels/jit/jit_lmc.mojo:275-330, lmc_provider.mojo:113-192)
  gradients  kernel params through A_s (x) dK_s; A_s and per-task noise
             (jit_lmc.mojo:582-691); NLL / SLQ as combined_inv_quad_logdet.mojo:452
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


def lmc_bbmm(specs, params_list, X, Y_centered, A, noise, num_probes, max_cg, max_tridiag, tol,
             iteration=0):
    """Y_centered [n, T]. Returns nll, kernel grads (concatenated), grad_A, grad_noise."""
    X = np.asarray(X, np.float64)
    n = X.shape[0]
    A = np.asarray(A, np.float64)
    T = A.shape[1]
    nT = n * T
    y = np.asarray(Y_centered, np.float64).T.reshape(nT)  # task-blocked
    K, Ks, Gs = full_operator(specs, params_list, X, A, np.asarray(noise, np.float64))
    seed = iteration * 104729 + 42
    W = ob.gaussian_block(nT, num_probes, seed)
    pn = np.linalg.norm(W, axis=0)
    rhs = np.concatenate([y[:, None], W / pn], axis=1)
    rn = np.linalg.norm(rhs, axis=0)
    x, iters, dg, od = ob.mbcg(K, rhs / rn, max_cg, max_tridiag, tol)
    sol = x * rn
    alpha = sol[:, 0]
    U = sol[:, 1:] * pn
    inv_quad = float(y @ alpha)
    logdet = ob.slq_logdet(dg[1:], od[1:], nT)
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
            "sum_alpha": sum_alpha, "cg_iters": iters, "K": K}
