"""Float64 restatement of the reference's training-side algorithms.

  hash_gaussian            kernels/pivoted_cholesky.mojo:51-86
  greedy pivoted Cholesky  kernels/pivoted_cholesky.mojo:2104-2444 (precond_method=0),
                           Woodbury 1646-1766, log|P| 1411-1517, probes 1909-2011
  mBCG                     kernels/combined_inv_quad_logdet.mojo:81-445
                           (+ cg_solver.mojo:108-250 freeze rules)
  tridiagonals + SLQ       combined_inv_quad_logdet.mojo:356-423,
                           native_numerics.mojo:403-518
  BBMM NLL / gradients     combined_inv_quad_logdet.mojo:452-1136
  Adam training loop       kernels/jit/jit_training.mojo:274-1008,
                           training_utils.mojo:23-315, utils.mojo:14-84

Arithmetic is float64 except where the reference's control flow depends on
float32 thresholds (1e-10, 1e-20, ...), which are applied to the same
quantities.
"""
from __future__ import annotations

import math

import numpy as np

from . import kernels as ok

M64 = (1 << 64) - 1


def hash_gaussian(idx: np.ndarray, seed: int) -> np.ndarray:
    """Counter-hash Box-Muller Gaussians of pivoted_cholesky.mojo:51-86."""
    idx = np.asarray(idx, dtype=np.uint64)
    with np.errstate(over="ignore"):
        s1 = (idx + np.uint64(1)) * np.uint64(6364136223846793005) + np.uint64(seed & M64)
        s1 ^= s1 >> np.uint64(33)
        s1 *= np.uint64(0xFF51AFD7ED558CCD)
        s1 ^= s1 >> np.uint64(33)
        s2 = (idx + np.uint64(1)) * np.uint64(1442695040888963407) + np.uint64(seed & M64) \
            + np.uint64(0xBEEF)
        s2 ^= s2 >> np.uint64(33)
        s2 *= np.uint64(0xC4CEB9FE1A85EC53)
        s2 ^= s2 >> np.uint64(33)
    u1 = ((s1 & np.uint64(0x7FFFFF)).astype(np.float64) + 1.0) / float(0x800000)
    u2 = (s2 & np.uint64(0xFFFFFF)).astype(np.float64) / float(0x1000000)
    two_pi = float(np.float32(2.0) * np.float32(3.14159265))
    return np.sqrt(-2.0 * np.log(u1)) * np.cos(two_pi * u2)


def gaussian_block(n: int, t: int, seed: int) -> np.ndarray:
    """[n, t] block whose column c holds indices c*n + i (column-major layout)."""
    idx = np.arange(n * t, dtype=np.uint64)
    return hash_gaussian(idx, seed).reshape(t, n).T.copy()


class Precond:
    """Greedy pivoted Cholesky P = L L^T + noise I (precond_method = 0)."""

    def __init__(self, K: np.ndarray, noise: float, rank: int, dtype=np.float64):
        """`dtype` = np.float32 repeats the factorisation in the reference's float32
        arithmetic (pivoted_cholesky.mojo is FP32); its trailing columns, where the
        residual diagonal is tiny, carry mostly rounding and shift log|P| visibly."""
        n = K.shape[0]
        K = np.asarray(K, dtype)
        diag = np.diag(K).astype(dtype).copy()
        mask = np.ones(n, dtype=bool)
        L = np.zeros((n, rank), dtype)
        pivots = []
        actual = rank
        for m in range(rank):
            cand = np.where(mask, diag, -np.inf)
            piv = int(np.argmax(cand))  # first maximal index = lowest index on ties
            maxv = cand[piv]
            if not (maxv >= 1e-10):
                actual = max(m, 1)
                break
            mask[piv] = False
            col = K[:, piv] - L[:, :m] @ L[piv, :m]
            col = col / dtype(math.sqrt(max(maxv, 1e-10)))
            L[:, m] = col
            diag[mask] -= col[mask] ** 2
            pivots.append(piv)
        self.L = L[:, :actual].astype(np.float64)
        self.rank = actual
        self.pivots = pivots
        self.noise = float(noise)
        M = self.L.T @ self.L
        eff = max(self.noise, 1e-6)
        self.Minv = np.linalg.inv(M + eff * np.eye(actual))
        _, ld = np.linalg.slogdet(np.eye(actual) + M / self.noise)
        self.logdet = n * math.log(self.noise) + ld

    def apply(self, V: np.ndarray) -> np.ndarray:
        return (V - self.L @ (self.Minv @ (self.L.T @ V))) / self.noise

    def sample(self, num: int, seed: int) -> np.ndarray:
        n = self.L.shape[0]
        zr = hash_gaussian(np.arange(self.rank * num, dtype=np.uint64), seed).reshape(num, self.rank).T
        zn = gaussian_block(n, num, seed + 1000000)
        return self.L @ zr + math.sqrt(self.noise) * zn


def greedy_pivots(column, diag0: np.ndarray, rank: int, follow=None, dtype=np.float32) -> dict:
    """The greedy pivot sequence of pivoted_cholesky.mojo:500-609 (argmax of
    the residual diagonal over unused rows, lowest index on ties,
    :537-539 / 573-577) and 772-1050 (stop below 1e-10; L[:, m] =
    (K[:, piv] - L[:, :m] L[piv, :m]^T) / sqrt(d_piv); d -= L[:, m]^2 on
    unused rows), with K given column by column: column(i) -> K[:, i].

    With `follow` (a pivot list, e.g. the GPU's), step m records its own
    argmax and then continues with follow[m], so every later step is checked
    against the same residual diagonal the follower saw. Per step it returns
    the own argmax `pivots`, its value, the followed pivot's value and `gap` =
    (own value - followed value) / own value (0 when they agree)."""
    n = diag0.shape[0]
    diag = np.asarray(diag0, dtype).copy()
    mask = np.ones(n, dtype=bool)
    L = np.zeros((n, rank), dtype)
    own, own_val, fol_val, gap = [], [], [], []
    steps = rank if follow is None else min(rank, len(follow))
    for m in range(steps):
        cand = np.where(mask, diag, -np.inf)
        piv = int(np.argmax(cand))
        maxv = float(cand[piv])
        if not (maxv >= 1e-10):
            break
        own.append(piv)
        own_val.append(maxv)
        use = piv if follow is None else int(follow[m])
        uv = float(cand[use])
        fol_val.append(uv)
        gap.append(0.0 if use == piv else (maxv - uv) / maxv)
        mask[use] = False
        col = np.asarray(column(use), dtype) - L[:, :m] @ L[use, :m]
        col = col / dtype(math.sqrt(max(uv, 1e-10)))
        L[:, m] = col
        diag[mask] -= col[mask] ** 2
    return {"pivots": own, "values": np.asarray(own_val), "followed_values": np.asarray(fol_val),
            "gap": np.asarray(gap)}


def mbcg(A: np.ndarray, rhs: np.ndarray, max_iter: int, max_tridiag: int, tol: float,
         precond: Precond | None = None, x0: np.ndarray | None = None):
    """Batched preconditioned CG with tridiagonal capture (float64)."""
    n, t = rhs.shape
    Pinv = precond.apply if precond is not None else (lambda v: v)
    if x0 is not None:
        x = x0.copy()
        r = rhs - A @ x
    else:
        x = np.zeros_like(rhs)
        r = rhs.copy()
    z = Pinv(r)
    p = z.copy()
    rz_old = np.sum(r * z, axis=0)
    alphas, betas = [], []
    iters = 0
    for it in range(max_iter):
        iters = it + 1
        Ap = A @ p
        pAp = np.sum(p * Ap, axis=0)
        alpha = np.where(np.isnan(rz_old) | np.isnan(pAp) | (pAp < 1e-10), 0.0,
                         rz_old / np.where(pAp == 0, 1.0, pAp))
        live = (alpha != 0) & ~np.isnan(alpha)
        x[:, live] += alpha[live] * p[:, live]
        r[:, live] -= alpha[live] * Ap[:, live]
        z = Pinv(r)
        rz_new = np.sum(r * z, axis=0)
        ok_ = ~np.isnan(rz_old) & ~np.isnan(rz_new) & (rz_old >= 1e-20)
        beta = np.where(ok_, rz_new / (rz_old + 1e-20), 0.0)
        beta = np.where((beta < 0) | np.isnan(beta), 0.0, beta)
        rz_old = np.where(np.isnan(rz_new), 0.0, rz_new)
        p = np.where(beta == 0, z, z + beta * p)
        if it < max_tridiag:
            alphas.append(alpha.copy())
            betas.append(beta.copy())
        if it >= 10 and ((it + 1) % 10 == 0 or it == max_iter - 1):
            mean_res = np.mean(np.linalg.norm(r, axis=0))
            if mean_res < tol and it >= max_tridiag - 1:
                break
    # tridiagonals
    size = min(iters, max_tridiag)
    diag = [[] for _ in range(t)]
    off = [[] for _ in range(t)]
    update = True
    for k in range(size):
        if not update:
            break
        max_off = 0.0
        for c in range(t):
            ak = alphas[k][c]
            ar = 1.0 if ak < 1e-10 else 1.0 / ak
            dv = ar
            if k > 0:
                akm = alphas[k - 1][c]
                prev = 1.0 if akm < 1e-10 else 1.0 / akm
                bkm = betas[k - 1][c]
                dv += bkm * prev
                o = math.sqrt(max(bkm, 0.0)) * prev
                off[c].append(o)
                max_off = max(max_off, o)
            diag[c].append(dv)
        if k > 0 and max_off < 1e-6:
            update = False
    return x, iters, diag, off


def slq_logdet(diags, offs, n: int) -> float:
    total, valid = 0.0, 0
    for d, e in zip(diags, offs):
        m = len(d)
        if m == 0:
            continue
        T = np.diag(d) + np.diag(e, 1) + np.diag(e, -1)
        lam, V = np.linalg.eigh(T)
        clamp = max(lam.max(), 1e-10) * 1e-6
        keep = (lam >= 0) & (lam >= clamp)
        total += float(np.sum(V[0, keep] ** 2 * np.log(lam[keep])))
        valid += 1
    return 0.0 if valid == 0 else n * total / valid


def bbmm(spec, params, X, y_centered, noise: float, num_probes: int, max_cg: int,
         max_tridiag: int, tol: float, iteration: int = 0, precond_rank: int = 0,
         precond: Precond | None = None, x_prev: np.ndarray | None = None):
    """One BBMM evaluation; returns dict(nll, grads (P+1), logdet, inv_quad, ...)."""
    X = np.asarray(X, np.float64)
    n = X.shape[0]
    K, G = ok.kernel_matrix(spec, params, X, want_grad=True)
    A = K + noise * np.eye(n)
    if precond is None and precond_rank > 0:
        precond = Precond(K, noise, precond_rank)
    seed = iteration * 104729 + 42
    sampled = precond.sample(num_probes, seed) if precond is not None else \
        gaussian_block(n, num_probes, seed)
    pn = np.linalg.norm(sampled, axis=0)
    Z = sampled / pn
    rhs = np.concatenate([np.asarray(y_centered, np.float64)[:, None], Z], axis=1)
    rn = np.linalg.norm(rhs, axis=0)
    rhs = rhs / rn
    x0 = None
    if x_prev is not None:
        x0 = np.zeros_like(rhs)
        x0[:, 0] = x_prev
    x, iters, dg, od = mbcg(A, rhs, max_cg, max_tridiag, tol, precond, x0)
    sol = x * rn
    alpha = sol[:, 0]
    inv_quad = float(np.dot(y_centered, alpha))
    logdet = slq_logdet(dg[1:], od[1:], n) + (precond.logdet if precond is not None else 0.0)
    PI = float(np.float32(3.14159265358979323846))
    nll = (0.5 * inv_quad + 0.5 * logdet + 0.5 * n * math.log(2 * PI)) / n
    U = sol[:, 1:] * pn
    W = precond.apply(sampled) if precond is not None else sampled
    grads = []
    for g in G:
        data = alpha @ g @ alpha
        trace = np.sum(U * (g @ W))
        grads.append((-0.5 * data + 0.5 * trace / num_probes) / n)
    gn = (-0.5 * alpha @ alpha + 0.5 * np.sum(U * W) / num_probes) / n
    grads.append(gn)
    return {"nll": nll, "grads": np.array(grads), "logdet": logdet, "inv_quad": inv_quad,
            "alpha": alpha, "cg_iters": iters, "x_norm0": x[:, 0], "sum_alpha": float(alpha.sum()),
            "precond": precond}


# ------------------------------------------------------------------ training
def softplus(x):
    if x > 20:
        return x
    if x < -20:
        return math.exp(x)
    return math.log1p(math.exp(x))


def inv_softplus(y):
    if y > 20:
        return y
    if y < 1e-6:
        return math.log(y)
    return math.log(math.expm1(y))


def softplus_derivative(x):
    if x > 20:
        return 1.0
    if x < -20:
        return math.exp(x)
    return 1.0 / (1.0 + math.exp(-x))


def clip_gradient(g, m=100.0):
    if g != g or abs(g) > 1e30:
        return 0.0
    return max(-m, min(m, g))


def train(spec, params, X, y, noise, *, max_iterations=10, learning_rate=0.01, num_probes=10,
          max_cg_iter=100, cg_tol=1e-2, precond_rank=0, max_tridiag_iter=30,
          precond_rebuild_threshold=0.5, use_cosine_lr=False, learn_noise=True, init_mean=0.0,
          trainable_mask=None):
    """Adam over softplus-raw params / noise / constant mean (jit_training.mojo:274-1008)."""
    P = len(params)
    raw = [inv_softplus(float(p)) for p in params] + [inv_softplus(float(noise))]
    m = [0.0] * (P + 1)
    v = [0.0] * (P + 1)
    t_adam = 0
    raw_mean, m_mean, v_mean = float(init_mean), 0.0, 0.0
    best = None
    best_nll = 1e30
    lr = learning_rate
    last_rebuild = [float(p) for p in params]
    last_noise = float(noise)
    X = np.asarray(X, np.float64)
    y = np.asarray(y, np.float64)
    n = X.shape[0]

    def build(cons, nz):
        if precond_rank <= 0:
            return None
        K = ok.kernel_matrix(spec, cons, X)
        return Precond(K, nz, precond_rank)

    cons = [softplus(r) for r in raw[:P]]
    pc = build(cons, softplus(raw[P]))
    hist = []
    x_prev = None
    for it in range(max_iterations):
        cons = [softplus(r) for r in raw[:P]]
        nz = softplus(raw[P]) if learn_noise else 0.0
        if it > 0:
            mr = max(abs(c - l) / max(abs(l), 1e-8) for c, l in zip(cons, last_rebuild))
            if learn_noise:
                mr = max(mr, abs(nz - last_noise) / max(abs(last_noise), 1e-8))
            if mr > precond_rebuild_threshold:
                pc = build(cons, nz)
                last_rebuild = list(cons)
                last_noise = nz
        yc = y - raw_mean
        res = bbmm(spec, np.array(cons), X, yc, nz, num_probes, max_cg_iter, max_tridiag_iter,
                   cg_tol, iteration=it, precond=pc, x_prev=x_prev)
        x_prev = res["x_norm0"]
        nll = res["nll"]
        hist.append(nll)
        if nll < best_nll:
            best_nll = nll
            best = (list(raw), raw_mean, res["alpha"])
        eff = lr
        if use_cosine_lr:
            lr_min = learning_rate / 20
            eff = lr_min + 0.5 * (learning_rate - lr_min) * (1 + math.cos(math.pi * it / max_iterations))
        g = list(res["grads"][:P]) + [res["grads"][P] if learn_noise else 0.0]
        if trainable_mask is not None:
            g = [gi if (q == P or trainable_mask[q]) else 0.0 for q, gi in enumerate(g)]
        t_adam += 1
        for q in range(P + 1):
            gr = clip_gradient(g[q]) * softplus_derivative(raw[q])
            m[q] = 0.9 * m[q] + 0.1 * gr
            v[q] = 0.999 * v[q] + 0.001 * gr * gr
        for q in range(P + 1):
            mh = m[q] / (1 - 0.9 ** t_adam)
            vh = v[q] / (1 - 0.999 ** t_adam)
            raw[q] = max(-20.0, min(20.0, raw[q] - eff * mh / (math.sqrt(vh) + 1e-8)))
        mg = clip_gradient(-res["sum_alpha"] / n)
        m_mean = 0.9 * m_mean + 0.1 * mg
        v_mean = 0.999 * v_mean + 0.001 * mg * mg
        raw_mean -= eff * (m_mean / (1 - 0.9 ** t_adam)) / (math.sqrt(v_mean / (1 - 0.999 ** t_adam)) + 1e-8)
        if raw_mean != raw_mean or abs(raw_mean) > 1000:
            raw_mean = init_mean
    braw, bmean, balpha = best
    return {"params": np.array([softplus(r) for r in braw[:P]]),
            "noise": softplus(braw[P]) if learn_noise else 0.0, "mean": bmean,
            "final_nll": best_nll, "nll_history": np.array(hist), "alpha": balpha}
