"""Float64 restatement of the ICM multi-output training loop.

Follows train_multi_output_jit (mojogp/kernels/jit/jit_multi_output.mojo:128-817)
with the task covariance of TaskCovariance (kernels/task_covariance.mojo:168-205):

  K_full = os * (B (x) K_X) + diag(noise_t) (x) I_n,   B = W W^T + diag(softplus(raw_v))

  * W starts from the counter hash in [0.1, 0.5] (task_covariance.mojo:194-200),
    raw_v = 0, raw params / outputscale / noise are inverse softplus of the
    initial values, the per-task means start at the given values (:175-186);
  * per iteration one BBMM evaluation of the LMC operator with one latent and
    A = os * B (the FusedKroneckerProvider is that operator), recycling the
    previous data-column solution unless the preconditioner was rebuilt in
    the iteration (:398-403), with the relative-change rebuild rule over
    params, outputscale, noise and B (:336-379) and a rebuild-and-retry when
    CG hits its cap (:405-440); a capped CG stops the fit (:447-468);
  * gradients: kernel params from BBMM, the outputscale through A = os B
    (the provider's last gradient), G_B = clip(os * dNLL/dA, +-10)
    (:520-566), noise per task (:570-601), then Adam (beta 0.9 / 0.999,
    eps 1e-8) over [kernel params, os, noise, W, raw_v, means] in that order;
    W is updated row by row in place, and each row's gradient 2 G_B[s, :] W[:, r]
    reads the rows already updated in this iteration (:648-662); the mean
    gradient is clip(-sum alpha_t / (n T), +-100) (:675-687);
  * early stopping on the NLL with `early_stop_tol` / `early_stop_patience`
    (:714-743); the result is the best-NLL state (:750-775).

Test infrastructure only (tests, smoke checks).
"""
from __future__ import annotations

import math

import numpy as np

from . import lmc as olmc


def softplus(x: float) -> float:
    return x if x > 20 else math.log1p(math.exp(x))


def inv_softplus(y: float) -> float:
    return y if y > 20 else math.log(math.expm1(y))


def sigmoid(x: float) -> float:
    return 1.0 / (1.0 + math.exp(-x))


def initial_W(T: int, R: int, seed: int = 42) -> np.ndarray:
    """task_covariance.mojo:194-200: LCG of (seed ^ i * 2654435761), scaled to [0.1, 0.5]."""
    out = np.empty(T * R, np.float32)
    for i in range(T * R):
        state = (seed ^ (i * 2654435761)) & ((1 << 64) - 1)
        state = (state * 1103515245 + 12345) & 0x7FFFFFFF
        r = np.float32(state) / np.float32(0x7FFFFFFF)
        out[i] = np.float32(0.1) + r * np.float32(0.4)
    return out.reshape(T, R)


def icm_fit(spec, X, Y, params0, *, max_iterations: int, learning_rate: float = 0.05,
            task_rank: int = -1, num_probes: int = 10, max_cg: int = 200,
            max_tridiag: int = 30, cg_tol: float = 1e-2, precond_rank: int = 15,
            rebuild_threshold: float = 0.5, initial_noise: float = 0.1,
            initial_outputscale: float = 1.0, init_mean=None, trainable=None,
            early_stop_tol: float = 1e-4, early_stop_patience: int = 15) -> dict:
    X = np.asarray(X, np.float64)
    Y = np.asarray(Y, np.float64)
    n, T = Y.shape
    R = T if task_rank < 0 else task_rank
    P = len(params0)
    trainable = np.ones(P, bool) if trainable is None else np.asarray(trainable, bool)
    raw_p = np.array([inv_softplus(float(v)) for v in params0])
    raw_os = inv_softplus(initial_outputscale)
    raw_noise = np.array([inv_softplus(initial_noise)] * T)
    raw_mean = (Y.mean(axis=0) if init_mean is None
                else np.broadcast_to(np.asarray(init_mean, np.float64), (T,))).astype(np.float64).copy()
    W = initial_W(T, R).astype(np.float64)
    raw_v = np.zeros(T)
    m = np.zeros(P + 1 + T + T * R + T + T)
    v = np.zeros_like(m)
    t_step = 1

    def adam(idx, g):
        m[idx] = 0.9 * m[idx] + 0.1 * g
        v[idx] = 0.999 * v[idx] + 0.001 * g * g
        mh = m[idx] / (1 - 0.9 ** t_step)
        vh = v[idx] / (1 - 0.999 ** t_step)
        return learning_rate * mh / (math.sqrt(vh) + 1e-8)

    def task_B():
        return W @ W.T + np.diag([softplus(r) for r in raw_v])

    def build(params, os_, noise, B):
        Kx = olmc.ok.kernel_matrix(spec, params, X)
        return olmc.LmcPrecond([Kx], (os_ * B)[None], noise, precond_rank,
                               factor_dtype=np.float32)

    params = np.array([softplus(r) for r in raw_p])
    pc = None
    if precond_rank > 0:
        pc = build(params, softplus(raw_os), np.array([softplus(r) for r in raw_noise]), task_B())
    # The rebuild rule runs (and suppresses recycling) with or without a
    # preconditioner (:336-403).
    last = np.concatenate([params, [softplus(raw_os)],
                           [softplus(r) for r in raw_noise], task_B().ravel()])
    hist, cg_hist = [], []
    best, best_nll_seen, es_best, patience = None, 1e30, 1e30, 0
    x_prev = None
    converged = False
    rebuilds = 0
    for it in range(max_iterations):
        params = np.array([softplus(r) for r in raw_p])
        os_ = softplus(raw_os)
        noise = np.array([softplus(r) for r in raw_noise])
        B = task_B()
        rebuilt = False
        if it > 0:
            cur = np.concatenate([params, [os_], noise, B.ravel()])
            if np.max(np.abs(cur - last) / (np.abs(last) + 1e-8)) > rebuild_threshold:
                if precond_rank > 0:
                    pc = build(params, os_, noise, B)
                last = cur
                rebuilt = True
                rebuilds += 1
        yc = Y - raw_mean[None, :]
        A = (os_ * B)[None]
        recycle = x_prev if (it > 0 and not rebuilt) else None
        res = olmc.lmc_bbmm([spec], [params], X, yc, A, noise, num_probes, max_cg, max_tridiag,
                            cg_tol, iteration=it, precond=pc, x_prev=recycle)
        if res["cg_iters"] >= max_cg and pc is not None:
            pc = build(params, os_, noise, B)
            last = np.concatenate([params, [os_], noise, B.ravel()])
            rebuilds += 1
            res = olmc.lmc_bbmm([spec], [params], X, yc, A, noise, num_probes, max_cg,
                                max_tridiag, cg_tol, iteration=it, precond=pc)
        x_prev = res["x_norm0"]
        nll = res["nll"]
        hist.append(nll)
        cg_hist.append(res["cg_iters"])
        cg_ok = res["cg_iters"] < max_cg
        state = (raw_p.copy(), raw_os, raw_noise.copy(), raw_mean.copy(), W.copy(), raw_v.copy(),
                 B.copy(), res["alpha"].copy())
        if not cg_ok:
            if best is None:
                best, best_nll_seen = state, nll
            break
        if nll < best_nll_seen:
            best, best_nll_seen = state, nll
        gA = res["gA"][0]  # dNLL/dA, A = os B
        G_B = np.clip(os_ * gA, -10.0, 10.0)
        kg = res["kgrads"]
        idx = 0
        for q in range(P):
            if trainable[q]:
                raw_p[q] -= adam(idx, kg[q] * sigmoid(raw_p[q]))
            idx += 1
        g_os = float(np.sum(gA * B))  # d/dos of os (B (x) K_X): the provider's outputscale gradient
        raw_os -= adam(idx, g_os * sigmoid(raw_os))
        idx += 1
        for t in range(T):
            raw_noise[t] -= adam(idx, res["gnoise"][t] * sigmoid(raw_noise[t]))
            idx += 1
        for s in range(T):
            for r in range(R):
                gw = 2.0 * float(G_B[s, :] @ W[:, r])  # rows < s already updated
                W[s, r] -= adam(idx, gw)
                idx += 1
        for t in range(T):
            raw_v[t] -= adam(idx, G_B[t, t] * sigmoid(raw_v[t]))
            idx += 1
        for t in range(T):
            g = float(np.clip(-res["sum_alpha"][t] / (n * T), -100.0, 100.0))
            raw_mean[t] -= adam(idx, g)
            idx += 1
        t_step += 1
        if early_stop_tol > 0:
            if nll < es_best - early_stop_tol:
                es_best = nll
                patience = 0
            else:
                patience += 1
                if patience >= early_stop_patience:
                    converged = True
                    break
    raw_p, raw_os, raw_noise, raw_mean, W, raw_v, B, alpha = best
    return {"nll_history": np.array(hist), "cg_iterations": cg_hist,
            "params": np.array([softplus(r) for r in raw_p]), "outputscale": softplus(raw_os),
            "noise": np.array([softplus(r) for r in raw_noise]), "mean": raw_mean, "W": W,
            "raw_v": raw_v, "B": B, "alpha": alpha, "best_nll": best_nll_seen,
            "converged": converged, "rebuilds": rebuilds}
