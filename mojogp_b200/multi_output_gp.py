"""MultiOutputLMCGP: linear model of coregionalisation, matrix-free on B200.

Mirrors the reference's MultiOutputLMCGP (mojogp/multi_output_gp.py:3465-5835)
for the matrix-free route and its training loop train_lmc_jit
(mojogp/kernels/jit/jit_lmc.mojo:699-1529): per-latent kernels K_s sharing X,
coregionalisation A_s = L_s L_s^T + diag(v_s) with softplus diagonals, per-task
noise and per-task constant means, Adam with gradient clip 10, NLL per n*T.
mBCG is preconditioned by the sum-of-Kronecker Woodbury preconditioner
(lmc_preconditioner.mojo), rebuilt when a kernel parameter or a task noise has
moved by more than `precond_rebuild_threshold` relative to the last build
(jit_lmc.mojo:1047-1100). Predictive variances follow predict_lmc
(kernels/jit/jit_engine_lmc_bindings.mojo:1102-1395): per-latent LOVE
variances with the mean task noise, weighted by the squared row norms of A_s,
plus the task noise.
"""
from __future__ import annotations

import ctypes as C
import math
from dataclasses import dataclass
from typing import List, Optional

import numpy as np

from . import _lib
from .kernel import Kernel, KernelNode, make_ard_kernel
from .gp import _check_multi_output_data, _check_test_inputs, _check_training_controls
from .provider import Provider

_STR = {"rbf": Kernel.rbf, "matern12": Kernel.matern12, "matern32": Kernel.matern32,
        "matern52": Kernel.matern52, "periodic": Kernel.periodic, "rq": Kernel.rq,
        "linear": Kernel.linear, "polynomial": Kernel.polynomial}


def _sp(x):
    return float(np.where(x > 20, x, np.log1p(np.exp(np.minimum(x, 20)))))


def _isp(y):
    return y if y > 20 else (math.log(y) if y < 1e-6 else math.log(math.expm1(y)))


def _dsp(x):
    return 1.0 / (1.0 + math.exp(-x)) if x > -20 else math.exp(x)


@dataclass
class MultiOutputPredictionResult:
    """Multi-output prediction (MultiOutputPredictionResult,
    multi_output_gp.py:545-550): mean [m, T], variance and std [m, T] or None."""

    mean: np.ndarray
    variance: Optional[np.ndarray] = None
    std: Optional[np.ndarray] = None


def _named(kernel, params, pick) -> np.ndarray:
    """The entries of `params` whose names (kernel.get_param_names) satisfy `pick`."""
    names = kernel.get_param_names()
    return np.asarray([float(params[i]) for i, nm in enumerate(names) if pick(nm)], np.float32)


def _observed_noise_matrix(m: int, T: int, observation_noise) -> np.ndarray:
    """Explicit test-point noise [m, T] for observed multi-output prediction
    (_resolve_observed_noise_matrix, multi_output_gp.py:553-601; grouped test
    noise belongs to the grouped-noise models, which are not built)."""
    if observation_noise is None:
        raise ValueError("Observed multi-output prediction requires explicit observation_noise "
                         "or noise_group_test; training noise is not reused for new points")
    noise = np.ascontiguousarray(observation_noise, dtype=np.float32)
    if noise.shape != (m, T):
        raise ValueError(f"observation_noise must have shape ({m}, {T}), got {noise.shape}")
    if not np.all(np.isfinite(noise)):
        raise ValueError("observed prediction noise contains NaN or Inf values")
    if np.any(noise <= 0):
        raise ValueError("observed prediction noise values must be > 0")
    return noise


def _observed_output(latent: "MultiOutputPredictionResult", noise: np.ndarray,
                     return_var: bool, return_std: bool):
    """latent variance + test noise (_format_observed_prediction, multi_output_gp.py:604-625)."""
    var = std = None
    if latent.variance is not None:
        var = np.ascontiguousarray(latent.variance + noise, dtype=np.float32)
        std = np.sqrt(var)
    if return_var:
        return latent.mean, var
    if return_std:
        return latent.mean, std
    return MultiOutputPredictionResult(mean=latent.mean, variance=var, std=std)


class _ObservedPredictionMixin:
    """Members the two multi-output models share: is_trained / training_result
    (multi_output_gp.py:1396-1430, 4634-4671), score (2753-2788) and
    predict_latent / predict_observed (2693-2740, 5558-5609)."""

    @property
    def is_trained(self) -> bool:
        return getattr(self, "_lmc", None) is not None and \
            getattr(self, "nll_history", None) is not None

    @property
    def training_result(self):
        """The fitted model itself (its properties carry the result fields), or None."""
        return self if self.is_trained else None

    def score(self, X_test, Y_test) -> dict:
        """rmse, mae, r2 over all tasks and rmse_per_task of the predictive mean."""
        if not self.is_trained:
            raise RuntimeError("GP must be trained before scoring. Call fit() first.")
        Y = np.ascontiguousarray(Y_test, dtype=np.float32)
        mean = self.predict(X_test, variance_method="mean_only").mean
        res = Y - mean
        ss_res = float(np.sum(res ** 2))
        ss_tot = float(np.sum((Y - Y.mean(axis=0)) ** 2))
        return {"rmse": float(np.sqrt(np.mean(res ** 2))), "mae": float(np.mean(np.abs(res))),
                "r2": float(1.0 - ss_res / (ss_tot + 1e-10)),
                "rmse_per_task": np.sqrt(np.mean(res ** 2, axis=0))}

    def predict_latent(self, X_test, return_var: bool = False, return_std: bool = False,
                       variance_method: str = "love", **kwargs):
        return self.predict(X_test, return_var=return_var, return_std=return_std,
                            variance_method=variance_method, **kwargs)

    def predict_observed(self, X_test, observation_noise=None, noise_group_test=None,
                         return_var: bool = False, return_std: bool = False,
                         variance_method: str = "love", **kwargs):
        if noise_group_test is not None:
            raise NotImplementedError("noise_group_test needs a grouped-noise model, which is "
                                      "not built; pass observation_noise [m, T]")
        latent = self.predict(X_test, variance_method=variance_method, **kwargs)
        noise = _observed_noise_matrix(latent.mean.shape[0], latent.mean.shape[1],
                                       observation_noise)
        return _observed_output(latent, noise, return_var, return_std)


def _prediction_output(mean, var, return_var: bool, return_std: bool):
    """The multi-output predict return convention: (mean, std) with return_std,
    (mean, variance) with return_var (zeros when no variance was computed),
    otherwise a MultiOutputPredictionResult."""
    if not (return_var or return_std):
        return MultiOutputPredictionResult(
            mean=mean, variance=var, std=None if var is None else np.sqrt(np.maximum(var, 0)))
    if var is None:
        var = np.zeros_like(mean)
    if return_std:
        return mean, np.sqrt(np.maximum(var, 0))
    return mean, var


def build_lmc_initial_params_from_lengthscales(kernels, initial_lengthscales) -> np.ndarray:
    """Flat LMC initial parameters from lengthscales: each latent's lengthscale
    slots take the given values, every other parameter 1
    (_build_lmc_initial_params_from_lengthscales, multi_output_gp.py:231-284).
    Accepted shapes: (R,) when every latent has one lengthscale, (total,) in
    latent order, or (R, c) when every latent has c lengthscales."""
    values = np.asarray(initial_lengthscales, dtype=np.float32)
    idx = [[i for i, nm in enumerate(k.get_param_names())
            if nm.endswith("_lengthscale") or "_ls_" in nm] for k in kernels]
    counts = [len(ix) for ix in idx]
    total = sum(counts)
    R = len(kernels)
    if total == 0:
        raise ValueError("initial_lengthscales was provided, but no latent has lengthscale parameters")
    if values.shape == (R,) and all(c == 1 for c in counts):
        per = [values[s:s + 1] for s in range(R)]
    elif values.shape == (total,):
        per, off = [], 0
        for c in counts:
            per.append(values[off:off + c])
            off += c
    elif len(set(counts)) == 1 and values.shape == (R, counts[0]):
        per = [values[s] for s in range(R)]
    else:
        shapes = [f"({total},)"]
        if all(c == 1 for c in counts):
            shapes.append(f"({R},)")
        if len(set(counts)) == 1:
            shapes.append(f"({R}, {counts[0]})")
        raise ValueError("initial_lengthscales must have shape " + " or ".join(shapes)
                         + f" for per-latent lengthscale counts {counts}, got {values.shape}")
    out = []
    for k, ix, vals in zip(kernels, idx, per):
        p = np.ones(k.num_params(), dtype=np.float32)
        p[ix] = vals
        out.append(p)
    return np.concatenate(out).astype(np.float32)


def _split_latent_params(kernels, initial_params, initial_lengthscales) -> list:
    """Per-latent starting parameters: the kernels' defaults, or a flat vector
    (given, or built from lengthscales) split in latent order."""
    if initial_params is None and initial_lengthscales is None:
        return [k.get_initial_params() for k in kernels]
    if initial_params is None:
        flat = build_lmc_initial_params_from_lengthscales(kernels, initial_lengthscales)
    else:
        flat = np.asarray(initial_params, dtype=np.float32).ravel()
    sizes = [k.num_params() for k in kernels]
    if flat.shape[0] != sum(sizes):
        raise ValueError(f"initial_params has {flat.shape[0]} values, expected {sum(sizes)} "
                         f"(per-latent counts {sizes})")
    if not np.all(np.isfinite(flat)) or np.any(flat <= 0):
        raise ValueError("initial parameters must be finite and > 0")
    out, off = [], 0
    for sz in sizes:
        out.append(flat[off:off + sz].copy())
        off += sz
    return out


class LMC:
    """Thin owner of a gpb_lmc handle over R providers."""

    def __init__(self, providers: List[Provider], num_tasks: int, comm=None):
        """comm: a distributed.Communicator to shard the data rows over the ranks
        (all tasks of a row on one GPU); host-side arrays stay full on every rank."""
        self.providers = providers
        self.T = num_tasks
        self.R = len(providers)
        self.n = providers[0].n
        self.comm = comm
        if comm is not None and comm.world > 1:
            from .distributed import shard_bounds
            self.r0, self.r1 = shard_bounds(self.n, comm.world, comm.rank)
        else:
            self.r0, self.r1 = 0, self.n
        arr = (C.c_void_p * self.R)(*[p.handle for p in providers])
        h = C.c_void_p()
        _lib.call("gpb_lmc_create_sharded", C.cast(arr, C.c_void_p), self.R, num_tasks,
                  C.c_void_p(comm.handle) if comm is not None else None, C.byref(h))
        self.handle = h.value

    def set_coregion(self, A: np.ndarray, noise: np.ndarray) -> None:
        A = np.ascontiguousarray(A, np.float32)
        nz = np.ascontiguousarray(noise, np.float32)
        _lib.call("gpb_lmc_set_coregion", C.c_void_p(self.handle), C.c_void_p(A.ctypes.data),
                  C.c_void_p(nz.ctypes.data))

    def bbmm(self, y_blocked: np.ndarray, num_probes: int, max_cg: int, max_tridiag: int,
             tol: float, iteration: int, recycle: bool):
        y = np.ascontiguousarray(y_blocked, np.float32).ravel()
        nll = C.c_double()
        P = sum(p.num_params for p in self.providers)
        kg = np.zeros(P)
        gA = np.zeros((self.R, self.T, self.T))
        gn = np.zeros(self.T)
        sa = np.zeros(self.T)
        alpha = np.zeros(self.n * self.T, np.float32)
        it = C.c_int32()
        _lib.call("gpb_lmc_bbmm", C.c_void_p(self.handle), C.c_void_p(y.ctypes.data), num_probes,
                  max_cg, max_tridiag, float(tol), iteration, int(recycle), C.byref(nll),
                  C.c_void_p(kg.ctypes.data), C.c_void_p(gA.ctypes.data),
                  C.c_void_p(gn.ctypes.data), C.c_void_p(sa.ctypes.data),
                  C.c_void_p(alpha.ctypes.data), C.byref(it))
        return {"nll": nll.value, "kgrads": kg, "gA": gA, "gnoise": gn, "sum_alpha": sa,
                "alpha": alpha, "cg_iters": it.value}

    def build_precond(self, rank: int):
        """Build (rank > 0) or remove (rank <= 0) the LMC preconditioner from the
        current A_s, noise and latent kernels; returns (per-latent ranks, log|P|)."""
        ranks = np.zeros(self.R, np.int32)
        ld = C.c_double()
        _lib.call("gpb_lmc_build_precond", C.c_void_p(self.handle), int(rank),
                  ranks.ctypes.data_as(C.POINTER(C.c_int32)), C.byref(ld))
        return ranks, ld.value

    def precond_apply_host(self, V: np.ndarray) -> np.ndarray:
        """P^{-1} V for task-blocked columns V [ncols, T*n_local] (this rank's rows)."""
        from .provider import DeviceBuffer
        V = np.ascontiguousarray(V, np.float32).reshape(-1, self.T * (self.r1 - self.r0))
        vd = DeviceBuffer.from_host(V, self.providers[0].device)
        od = DeviceBuffer(V.shape, self.providers[0].device)
        _lib.call("gpb_lmc_precond_apply", C.c_void_p(self.handle), od.cptr, vd.cptr, V.shape[0])
        return od.download()

    def precond_sample_host(self, num: int, seed: int) -> np.ndarray:
        from .provider import DeviceBuffer
        od = DeviceBuffer((num, self.T * (self.r1 - self.r0)), self.providers[0].device)
        _lib.call("gpb_lmc_precond_sample", C.c_void_p(self.handle), od.cptr, int(num),
                  C.c_uint64(seed))
        return od.download()

    def solve(self, rhs: np.ndarray, max_cg: int = 300, tol: float = 1e-3):
        r = np.ascontiguousarray(rhs, np.float32).ravel()
        x = np.zeros_like(r)
        it = C.c_int32()
        _lib.call("gpb_lmc_solve", C.c_void_p(self.handle), C.c_void_p(r.ctypes.data), max_cg,
                  float(tol), C.c_void_p(x.ctypes.data), C.byref(it))
        return x, it.value

    def exact_variance(self, X_test: np.ndarray, max_cg: int = 100, tol: float = 1e-2,
                       block_cols: int = 0):
        """Exact posterior variance [m, T] of every task at X_test (observation
        noise included); returns (variance, total CG iterations)."""
        Xt = np.ascontiguousarray(X_test, np.float32)
        m = Xt.shape[0]
        var = np.zeros((m, self.T), np.float32)
        it = C.c_int32()
        _lib.call("gpb_lmc_predict_exact_variance", C.c_void_p(self.handle),
                  C.c_void_p(Xt.ctypes.data), m, int(block_cols), int(max_cg), float(tol),
                  C.c_void_p(var.ctypes.data), C.byref(it))
        return var, it.value

    def destroy(self) -> None:
        if getattr(self, "handle", None):
            _lib.lib().gpb_lmc_destroy(C.c_void_p(self.handle))
            self.handle = None

    def __del__(self):
        try:
            self.destroy()
        except Exception:
            pass


class MultiOutputLMCGP(_ObservedPredictionMixin):
    """LMC multi-output GP with heterogeneous latent kernels."""

    def __init__(self, kernels: list, num_probes: int = 10, max_cg_iterations: int = 200,
                 cg_tolerance: float = 1.0, max_tridiag_iterations: int = 30, ard: bool = False,
                 init_mean=None, device: int = 0, preconditioner_rank: int = 15,
                 precond_rebuild_threshold: float = 0.5, lanczos_rank: int = 0):
        ks = []
        for k in kernels:
            if isinstance(k, str):
                if k.lower() not in _STR:
                    raise ValueError(f"Unknown kernel '{k}'. Must be one of: {list(_STR)}")
                k = _STR[k.lower()]()
            if not isinstance(k, KernelNode):
                raise ValueError(f"All kernels must be KernelNode objects or kernel strings, got {type(k)}")
            ks.append(k)
        if not ks:
            raise ValueError("need at least one latent kernel")
        self.kernels = ks
        self.num_latents = len(ks)
        self.num_probes = num_probes
        self.max_cg_iter = max_cg_iterations
        self.cg_tol = cg_tolerance
        self.max_tridiag_iter = max_tridiag_iterations
        self.ard = ard
        self.init_mean = init_mean
        self.device = device
        self.precond_rank = int(preconditioner_rank)
        self.precond_rebuild_threshold = float(precond_rebuild_threshold)
        self.lanczos_rank = int(lanczos_rank)
        self._lmc: Optional[LMC] = None

    def _state_to_A(self, L, raw_L_diag, raw_var):
        R, T = self.num_latents, self.T
        A = np.zeros((R, T, T))
        L = L.copy()
        for s in range(R):
            for i in range(T):
                L[s, i, i] = _sp(raw_L_diag[s, i])
            A[s] = L[s] @ L[s].T + np.diag([_sp(v) for v in raw_var[s]])
        return A, L

    def fit(self, X, Y, max_iterations: int = 100, learning_rate: float = 0.05,
            initial_noise: float = 0.1, method: str = "matrix_free", verbose: bool = False,
            initial_params=None, initial_lengthscales=None, comm=None):
        """initial_params: the latents' public parameters concatenated in
        latent order; initial_lengthscales: lengthscales only, the other
        parameters at 1 (_build_lmc_initial_params_from_lengthscales,
        multi_output_gp.py:231-284); at most one of the two."""
        if method not in ("matrix_free", "mf", "auto", "materialized", "mat"):
            raise ValueError(f"method={method!r}: expected 'matrix_free' or 'materialized'")
        # "materialized" is served by the matrix-free operator (see SingleOutputGP.fit).
        X = np.ascontiguousarray(X, np.float32)
        Y = np.asarray(Y, np.float32)
        _check_multi_output_data(X, Y)
        _check_training_controls(max_iterations, learning_rate, initial_noise)
        if initial_params is not None and initial_lengthscales is not None:
            raise ValueError("Provide initial_params or initial_lengthscales, not both")
        n, d = X.shape
        T = Y.shape[1]
        R = self.num_latents
        self.kernels_resolved = [make_ard_kernel(k, d) if self.ard else k.resolve_ard(d)
                                 for k in self.kernels]
        params0 = _split_latent_params(self.kernels_resolved, initial_params, initial_lengthscales)
        self.T, self.dim = T, d
        self._X = X
        masks = [k.engine_trainable_mask() for k in self.kernels_resolved]
        provs = [Provider(X, k, p, 0.0, device=self.device)
                 for k, p in zip(self.kernels_resolved, params0)]
        self._lmc = LMC(provs, T, comm=comm)
        raw_p = [np.array([_isp(float(v)) for v in p]) for p in params0]
        raw_noise = np.array([_isp(initial_noise)] * T)
        if self.init_mean is None:
            raw_mean = Y.mean(axis=0).astype(np.float64)
        else:
            raw_mean = np.broadcast_to(np.asarray(self.init_mean, np.float64), (T,)).copy()
        init_diag = math.sqrt(1.0 / R)
        L = np.zeros((R, T, T))
        for s in range(R):
            for i in range(T):
                for j in range(i):
                    L[s, i, j] = 0.01 * (s + 1) / R
        raw_L_diag = np.full((R, T), _isp(init_diag))
        raw_var = np.full((R, T), _isp(0.1))
        sizes = [len(p) for p in raw_p]
        n_adam = sum(sizes) + T + R * T * T + R * T + T
        m = np.zeros(n_adam)
        v = np.zeros(n_adam)
        clip = lambda g: float(np.clip(g, -10.0, 10.0)) if np.isfinite(g) else 0.0
        Yb = Y.T.astype(np.float64)  # [T, n] task-blocked
        best = None
        hist = []
        cg_hist = []
        t_step = 0
        last_build = None  # (kernel params, noise) at the last preconditioner build
        self.precond_rebuild_count = 0
        self.precond_ranks = None

        def adam(idx, g):
            m[idx] = 0.9 * m[idx] + 0.1 * g
            v[idx] = 0.999 * v[idx] + 0.001 * g * g
            mh = m[idx] / (1 - 0.9 ** t_step)
            vh = v[idx] / (1 - 0.999 ** t_step)
            return -learning_rate * mh / (math.sqrt(vh) + 1e-8)

        for it in range(max_iterations):
            t_step += 1
            for s in range(R):
                provs[s].update_params(np.array([_sp(r) for r in raw_p[s]], np.float32))
            A, Lf = self._state_to_A(L, raw_L_diag, raw_var)
            noise = np.array([_sp(r) for r in raw_noise])
            self._lmc.set_coregion(A, noise)
            if self.precond_rank > 0:
                cur = (np.concatenate([[_sp(r) for r in rp] for rp in raw_p]), noise.copy())
                rebuild = last_build is None
                if not rebuild:
                    rel = [np.max(np.abs(c - l) / (np.abs(l) + 1e-8)) if c.size else 0.0
                           for c, l in zip(cur, last_build)]
                    rebuild = max(rel) > self.precond_rebuild_threshold
                if rebuild:
                    if last_build is not None:
                        self.precond_rebuild_count += 1
                    self.precond_ranks, _ = self._lmc.build_precond(self.precond_rank)
                    last_build = cur
            yc = (Yb - raw_mean[:, None]).astype(np.float32)
            res = self._lmc.bbmm(yc, self.num_probes, self.max_cg_iter, self.max_tridiag_iter,
                                 self.cg_tol, it, it > 0)
            nll = res["nll"]
            hist.append(nll)
            cg_hist.append(res["cg_iters"])
            if not np.isfinite(nll):
                if best is None:
                    raise FloatingPointError("LMC NLL is not finite at the initial parameters")
                raw_p, raw_noise, raw_mean, L, raw_L_diag, raw_var = [np.copy(x) if not isinstance(x, list) else [np.copy(y) for y in x] for x in best[1:7]]
                raw_var = raw_var + 0.7
                continue
            if best is None or nll < best[0]:
                best = (nll, [np.copy(r) for r in raw_p], raw_noise.copy(), raw_mean.copy(),
                        L.copy(), raw_L_diag.copy(), raw_var.copy())
            idx = 0
            off = 0
            for s in range(R):
                for q in range(sizes[s]):
                    if masks[s][q]:
                        g = clip(res["kgrads"][off + q]) * _dsp(raw_p[s][q])
                        raw_p[s][q] += adam(idx, g)
                    idx += 1
                off += sizes[s]
            for t in range(T):
                raw_noise[t] += adam(idx, clip(res["gnoise"][t]) * _dsp(raw_noise[t]))
                idx += 1
            gA = res["gA"]
            for s in range(R):
                for i in range(T):
                    for j in range(i + 1):
                        gL = clip(2.0 * float(gA[s, i, :] @ Lf[s][:, j]))
                        if i == j:
                            raw_L_diag[s, i] += adam(idx, gL * _dsp(raw_L_diag[s, i]))
                        else:
                            L[s, i, j] += adam(idx, gL)
                        idx += 1
                    idx += T - i - 1
            for s in range(R):
                for i in range(T):
                    raw_var[s, i] += adam(idx, clip(gA[s, i, i]) * _dsp(raw_var[s, i]))
                    idx += 1
            for t in range(T):
                raw_mean[t] += adam(idx, clip(-res["sum_alpha"][t] / (n * T)))
                idx += 1
            if verbose and (it < 5 or it % 10 == 0):
                print(f"LMC iter {it}: NLL = {nll:.6f}")
        _, raw_p, raw_noise, raw_mean, L, raw_L_diag, raw_var = best
        for s in range(R):
            provs[s].update_params(np.array([_sp(r) for r in raw_p[s]], np.float32))
        A, _ = self._state_to_A(L, raw_L_diag, raw_var)
        noise = np.array([_sp(r) for r in raw_noise])
        self._lmc.set_coregion(A, noise)
        self.A, self.noise, self.mean_ = A, noise, raw_mean
        self.params_ = [np.array([_sp(r) for r in rp]) for rp in raw_p]
        self.nll_history = np.array(hist)
        self.cg_iterations_history = cg_hist
        self.final_nll = best[0]
        yc = (Yb - raw_mean[:, None]).astype(np.float32)
        self._alpha, _ = self._lmc.solve(yc, 300, 1e-3)
        return self

    # Training-result fields (LMCTrainingResult, multi_output_gp.py:3405-3464): fit()
    # returns the model, which answers for the result object.
    @property
    def num_tasks(self) -> int:
        return self.T

    @property
    def iterations(self) -> int:
        return len(self.nll_history)

    @property
    def converged(self) -> bool:
        return False  # the LMC loop runs its iteration budget

    @property
    def noise_per_task(self) -> np.ndarray:
        return np.asarray(self.noise)

    @property
    def params_per_latent(self) -> list:
        return [np.asarray(p) for p in self.params_]

    @property
    def task_covariance(self) -> Optional[np.ndarray]:
        """B = sum_s A_s [T, T], None before fit (multi_output_gp.py:4659-4663)."""
        return self.B if getattr(self, "A", None) is not None else None

    @property
    def A_matrices(self) -> np.ndarray:
        return np.asarray(self.A)

    @property
    def B(self) -> np.ndarray:
        return np.asarray(self.A).sum(axis=0)

    @property
    def Lambda(self) -> np.ndarray:
        return np.linalg.eigh(self.B)[0]

    @property
    def Q(self) -> np.ndarray:
        return np.linalg.eigh(self.B)[1]

    @property
    def alpha(self) -> np.ndarray:
        """[n, T] solution of K_full alpha = y - mean (task-blocked internally)."""
        return self._alpha.reshape(self.T, -1).T

    @property
    def mean_per_task(self) -> np.ndarray:
        return np.asarray(self.mean_)

    @property
    def use_ard(self) -> bool:
        return bool(self.ard)

    @property
    def lengthscales(self) -> np.ndarray:
        """Every latent's lengthscale parameters, in latent order."""
        return np.concatenate([_named(k, p, lambda nm: nm.endswith("_lengthscale") or "_ls_" in nm)
                               for k, p in zip(self.kernels_resolved, self.params_)])

    @property
    def outputscales(self) -> np.ndarray:
        return np.concatenate([_named(k, p, lambda nm: nm.endswith("_outputscale"))
                               for k, p in zip(self.kernels_resolved, self.params_)])

    def log_marginal_likelihood(self) -> float:
        return -float(self.final_nll)

    def predict(self, X_test, return_var: bool = False, return_std: bool = False,
                variance_method: str = "love"):
        """Mean [m, T]; with return_var / return_std also the variance / std [m, T]
        (observation noise included). variance_method (MultiOutputLMCGP.predict,
        mojogp/multi_output_gp.py:5406-5556): 'love' sums per-latent LOVE
        variances weighted by the row norms of A_s; 'exact' is the full LMC
        posterior diagonal by batched CG (_predict_lmc_full_exact_variance_backend,
        4360-4519, with CG iterations max(max_cg_iterations, 100) and tolerance
        min(cg_tolerance, 1e-2)); 'mean_only' returns zero variance."""
        if self._lmc is None:
            raise RuntimeError("GP must be trained before prediction. Call fit() first.")
        if variance_method not in ("love", "exact", "mean_only"):
            raise ValueError("variance_method must be one of ('love', 'exact', 'mean_only'), "
                             f"got '{variance_method}'")
        Xt = np.ascontiguousarray(X_test, np.float32)
        if Xt.ndim == 1 and self.dim == 1:
            Xt = Xt[:, None]
        _check_test_inputs(Xt, self.dim)
        mean = self._predict_mean(Xt)
        var = None if variance_method == "mean_only" else self._predict_var(Xt, variance_method)
        return _prediction_output(mean, var, return_var, return_std)

    def _predict_mean(self, Xt: np.ndarray) -> np.ndarray:
        T, n = self.T, self._X.shape[0]
        alpha = self._alpha.reshape(T, n).T  # [n, T]
        mean = np.zeros((Xt.shape[0], T))
        for s, prov in enumerate(self._lmc.providers):
            Cs = prov.cross_matvec_host(Xt, alpha)  # [n*, T] = K_s(X*, X) alpha_j
            mean += Cs @ self.A[s].T
        return (mean + self.mean_[None, :]).astype(np.float32)

    def _predict_var(self, Xt: np.ndarray, variance_method: str) -> np.ndarray:
        T, n = self.T, self._X.shape[0]
        if variance_method == "exact":
            tol = min(float(self.cg_tol), 1e-2) if self.cg_tol > 0 else 1e-2
            var, _ = self._lmc.exact_variance(Xt, max(int(self.max_cg_iter), 100), tol)
            return var
        from .gp import _DEFAULT_PREDICT_LANCZOS_RANK
        from .prediction import PredictionCache
        avg_noise = float(np.mean(self.noise))
        var = np.zeros((Xt.shape[0], T))
        for s, prov in enumerate(self._lmc.providers):
            rank = self.lanczos_rank
            if rank <= 0:
                ard = self.kernels_resolved[s].has_ard()
                rank = max(_DEFAULT_PREDICT_LANCZOS_RANK, 200 if ard else 0)
            rank = min(rank, n)
            prov.update_noise(avg_noise)
            try:
                cache = PredictionCache(prov, np.zeros(n, np.float32), 0.0, rank)
                _, v_s = cache.predict(Xt, return_var=True)
                cache.destroy()
            finally:
                prov.update_noise(0.0)
            latent = np.maximum(v_s.astype(np.float64) - avg_noise, 1e-10)
            row_w = (self.A[s] ** 2).sum(axis=1)  # sum_t' A_s[t][t']^2
            var += latent[:, None] * row_w[None, :]
        return (var + self.noise[None, :]).astype(np.float32)


def _icm_initial_W(T: int, R: int, seed: int = 42) -> np.ndarray:
    """Initial low-rank task factor W [T, R] in [0.1, 0.5] from the reference's
    counter-hash (kernels/task_covariance.mojo:168-205): the same numbers, so a
    fit starts from the reference's state."""
    W = np.empty(T * R, np.float32)
    for i in range(T * R):
        state = (seed ^ ((i * 2654435761) & 0xFFFFFFFFFFFFFFFF)) & 0xFFFFFFFFFFFFFFFF
        state = (state * 1103515245 + 12345) & 0x7FFFFFFF
        W[i] = np.float32(0.1) + np.float32(np.float32(state) / np.float32(0x7FFFFFFF)) * np.float32(0.4)
    return W.reshape(T, R)


class MultiOutputGP(_ObservedPredictionMixin):
    """Multi-output GP with ICM task covariance, matrix-free on B200.

    Mirrors the reference's MultiOutputGP (mojogp/multi_output_gp.py:859-2520)
    and train_multi_output_jit (kernels/jit/jit_multi_output.mojo:128-817):
      K_full = os * (B (x) K_X) + diag(noise_t (x) 1_n),  B = W W^T + diag(softplus(raw_v)),
    i.e. the LMC operator with one latent kernel and A = os * B, trained by BBMM
    with the sum-of-Kronecker preconditioner (KroneckerPreconditioner is its R = 1
    case). Prediction follows predict_multi_output
    (jit_engine_multi_output_bindings.mojo:329-545): with os * B = Q Lambda Q^T
    (Lambda clamped at 1e-6) and mean task noise s2, the latent variance is
    sum_s Q[t, s]^2 lambda_s var_s(x*), var_s the posterior variance of K_X with
    noise s2 / lambda_s (LOVE or exact CG); the mean is K(X*, X) alpha (os B)^T + mean_t.
    """

    _PRESETS = {
        "fast": dict(max_cg_iter=50, cg_tol=5e-2, num_probes=5, max_tridiag_iter=15,
                     precond_rank=5, precond_rebuild_threshold=0.75),
        "balanced": dict(max_cg_iter=200, cg_tol=1e-2, num_probes=10, max_tridiag_iter=30,
                         precond_rank=15, precond_rebuild_threshold=0.5),
        "accurate": dict(max_cg_iter=400, cg_tol=1e-2, num_probes=20, max_tridiag_iter=60,
                         precond_rank=20, precond_rebuild_threshold=0.25),
    }

    def __init__(self, kernel="rbf", task_rank: int = -1, ard: bool = False,
                 num_probes: Optional[int] = None, max_cg_iterations: Optional[int] = None,
                 cg_tolerance: Optional[float] = None, preconditioner_rank: Optional[int] = None,
                 precond_rebuild_threshold: Optional[float] = None,
                 use_preconditioner: Optional[bool] = None, init_mean=None,
                 preset: Optional[str] = None, max_tridiag_iterations: Optional[int] = None,
                 device: int = 0):
        if preset is not None and preset not in self._PRESETS:
            raise ValueError(f"Unknown preset '{preset}'. Must be one of: {list(self._PRESETS)}")
        base = dict(self._PRESETS[preset or "balanced"])
        for key, val in (("num_probes", num_probes), ("max_cg_iter", max_cg_iterations),
                         ("cg_tol", cg_tolerance), ("precond_rank", preconditioner_rank),
                         ("precond_rebuild_threshold", precond_rebuild_threshold),
                         ("max_tridiag_iter", max_tridiag_iterations)):
            if val is not None:
                base[key] = val
        if use_preconditioner is False:
            base["precond_rank"] = 0
        if isinstance(kernel, str):
            if kernel.lower() not in _STR:
                raise ValueError(f"Unknown kernel '{kernel}'. Must be one of: {list(_STR)}")
            kernel = _STR[kernel.lower()]()
        if not isinstance(kernel, KernelNode):
            raise ValueError(f"kernel must be a KernelNode or a kernel string, got {type(kernel)}")
        self.kernel = kernel
        self.task_rank = int(task_rank)
        self.ard = ard
        self.num_probes = int(base["num_probes"])
        self.max_cg_iter = int(base["max_cg_iter"])
        self.cg_tol = float(base["cg_tol"])
        self.max_tridiag_iter = int(base["max_tridiag_iter"])
        self.precond_rank = int(base["precond_rank"])
        self.precond_rebuild_threshold = float(base["precond_rebuild_threshold"])
        self.init_mean = init_mean
        self.device = device
        self._lmc: Optional[LMC] = None

    # ------------------------------------------------------------------ fit
    def fit(self, X, Y, max_iterations: int = 100, learning_rate: float = 0.05,
            method: str = "materialized", initial_noise: float = 0.1,
            initial_noise_per_task=None, verbose: bool = False, early_stop_tol: float = 1e-4,
            early_stop_patience: int = 15, comm=None):
        if method not in ("matrix_free", "mf", "auto", "materialized", "mat"):
            raise ValueError(f"method={method!r}: expected 'matrix_free' or 'materialized'")
        # "materialized" is served by the matrix-free operator (see SingleOutputGP.fit).
        X = np.ascontiguousarray(X, np.float32)
        Y = np.asarray(Y, np.float32)
        _check_multi_output_data(X, Y)
        _check_training_controls(max_iterations, learning_rate, initial_noise)
        n, d = X.shape
        T = Y.shape[1]
        R = T if self.task_rank < 0 else self.task_rank
        if R < 1 or R > T:
            raise ValueError(f"task_rank must be -1 or in [1, {T}]")
        self.T, self.dim, self._X = T, d, X
        self.kernel_resolved = make_ard_kernel(self.kernel, d) if self.ard else \
            self.kernel.resolve_ard(d)
        params0 = np.asarray(self.kernel_resolved.get_initial_params(), np.float32)
        mask = np.asarray(self.kernel_resolved.engine_trainable_mask(), bool)
        prov = Provider(X, self.kernel_resolved, params0, 0.0, device=self.device)
        self._lmc = LMC([prov], T, comm=comm)
        raw_p = np.array([_isp(float(v)) for v in params0])
        raw_os = _isp(1.0)
        noise0 = (np.full(T, initial_noise) if initial_noise_per_task is None
                  else np.asarray(initial_noise_per_task, np.float64))
        raw_noise = np.array([_isp(float(v)) for v in noise0])
        if self.init_mean is None:
            raw_mean = Y.mean(axis=0).astype(np.float64)
        else:
            raw_mean = np.broadcast_to(np.asarray(self.init_mean, np.float64), (T,)).copy()
        W = _icm_initial_W(T, R).astype(np.float64)
        raw_v = np.zeros(T)
        P = len(raw_p)
        m = np.zeros(P + 1 + T + T * R + T + T)
        v = np.zeros_like(m)
        lr = learning_rate
        t_step = 1

        def adam(idx, g):
            m[idx] = 0.9 * m[idx] + 0.1 * g
            v[idx] = 0.999 * v[idx] + 0.001 * g * g
            mh = m[idx] / (1 - 0.9 ** t_step)
            vh = v[idx] / (1 - 0.999 ** t_step)
            return -lr * mh / (math.sqrt(vh) + 1e-8)

        Yb = Y.T.astype(np.float64)
        hist, cg_hist = [], []
        best, best_nll, patience = None, 1e30, 0
        es_best = 1e30  # early-stopping tracker, separate from the best state
        last = None
        self.precond_rebuild_count = 0
        converged = False
        for it in range(max_iterations):
            params = np.array([_sp(r) for r in raw_p], np.float32)
            prov.update_params(params)
            os_ = _sp(raw_os)
            noise = np.array([_sp(r) for r in raw_noise])
            B = W @ W.T + np.diag([_sp(r) for r in raw_v])
            self._lmc.set_coregion((os_ * B)[None].astype(np.float32), noise)
            state = (np.concatenate([params, [os_], noise, B.ravel()]))
            # The rebuild rule (jit_multi_output.mojo:336-379) runs with or
            # without a preconditioner; a rebuild iteration does not recycle
            # the previous solution (:398-403).
            rebuild = last is None or np.max(np.abs(state - last) /
                                             (np.abs(last) + 1e-8)) > self.precond_rebuild_threshold
            if rebuild:
                if last is not None:
                    self.precond_rebuild_count += 1
                if self.precond_rank > 0:
                    self._lmc.build_precond(self.precond_rank)
                last = state
            yc = (Yb - raw_mean[:, None]).astype(np.float32)
            res = self._lmc.bbmm(yc, self.num_probes, self.max_cg_iter, self.max_tridiag_iter,
                                 self.cg_tol, it, it > 0 and not rebuild)
            if res["cg_iters"] >= self.max_cg_iter and self.precond_rank > 0:
                # jit_multi_output.mojo: rebuild the preconditioner and retry once
                self._lmc.build_precond(self.precond_rank)
                last = state
                self.precond_rebuild_count += 1
                res = self._lmc.bbmm(yc, self.num_probes, self.max_cg_iter, self.max_tridiag_iter,
                                     self.cg_tol, it, False)
            nll = res["nll"]
            hist.append(nll)
            cg_hist.append(res["cg_iters"])
            cg_ok = res["cg_iters"] < self.max_cg_iter
            if (cg_ok or best is None) and np.isfinite(nll) and nll < best_nll:
                best_nll = nll
                best = (raw_p.copy(), raw_os, raw_noise.copy(), raw_mean.copy(), W.copy(),
                        raw_v.copy(), res["alpha"].copy())
            if not cg_ok:
                break  # stop with the best valid state (jit_multi_output.mojo)
            gA = res["gA"][0]
            G_B = np.clip(os_ * gA, -10.0, 10.0)
            sig = lambda x: 1.0 / (1.0 + math.exp(-x))
            idx = 0
            for q in range(P):
                if mask[q]:
                    raw_p[q] += adam(idx, res["kgrads"][q] * sig(raw_p[q]))
                idx += 1
            g_os = float(np.sum(gA * B))  # dNLL/dos through A = os B
            raw_os += adam(idx, g_os * sig(raw_os))
            idx += 1
            for t in range(T):
                raw_noise[t] += adam(idx, res["gnoise"][t] * sig(raw_noise[t]))
                idx += 1
            # Row by row in place: each row's gradient reads the rows already
            # updated in this iteration (jit_multi_output.mojo:648-662).
            for s in range(T):
                for r in range(R):
                    W[s, r] += adam(idx, 2.0 * float(G_B[s, :] @ W[:, r]))
                    idx += 1
            for t in range(T):
                raw_v[t] += adam(idx, G_B[t, t] * sig(raw_v[t]))
                idx += 1
            for t in range(T):
                g = float(np.clip(-res["sum_alpha"][t] / (n * T), -100.0, 100.0))
                raw_mean[t] += adam(idx, g)
                idx += 1
            t_step += 1
            if verbose and (it % 10 == 0 or it == max_iterations - 1):
                print(f"MO Iter {it}: NLL = {nll}")
            if early_stop_tol > 0:
                if nll < es_best - early_stop_tol:
                    es_best = nll
                    patience = 0
                else:
                    patience += 1
                    if patience >= early_stop_patience:
                        converged = True
                        break
        raw_p, raw_os, raw_noise, raw_mean, W, raw_v, alpha = best
        self.params_ = np.array([_sp(r) for r in raw_p], np.float32)
        prov.update_params(self.params_)
        self.outputscale_ = _sp(raw_os)
        self.noise_per_task = np.array([_sp(r) for r in raw_noise])
        self.mean_ = raw_mean
        self.W_ = W
        Bs = self.outputscale_ * (W @ W.T + np.diag([_sp(r) for r in raw_v]))
        self.task_covariance = Bs
        self._lmc.set_coregion(Bs[None].astype(np.float32), self.noise_per_task)
        ev, Q = np.linalg.eigh(Bs)
        self._Lambda = np.maximum(ev, 1e-6)
        self._Q = Q
        self._alpha = alpha
        self.nll_history = np.array(hist)
        self.cg_iterations_history = cg_hist
        self.final_nll = best_nll
        self.converged = converged
        return self

    # Training-result fields (MultiOutputTrainingResult, multi_output_gp.py:475-543):
    # fit() returns the model, which answers for the result object.
    @property
    def num_tasks(self) -> int:
        return self.T

    @property
    def iterations(self) -> int:
        return len(self.nll_history)

    @property
    def noise(self) -> float:
        return float(np.mean(self.noise_per_task))

    @property
    def params(self) -> np.ndarray:
        return np.asarray(self.params_)

    @property
    def num_kernel_params(self) -> int:
        return int(np.asarray(self.params_).shape[0])

    @property
    def B(self) -> np.ndarray:
        return self.task_covariance

    @property
    def Q(self) -> np.ndarray:
        return self._Q

    @property
    def Lambda(self) -> np.ndarray:
        return self._Lambda

    @property
    def effective_scales(self) -> np.ndarray:
        return self._Lambda

    @property
    def W(self) -> np.ndarray:
        return self.W_

    @property
    def mean_per_task(self) -> np.ndarray:
        return np.asarray(self.mean_)

    def log_marginal_likelihood(self) -> float:
        return -float(self.final_nll)

    # ------------------------------------------------------------ predict
    def predict(self, X_test, return_var: bool = False, return_std: bool = False,
                variance_method: str = "love", lanczos_rank: int = 0):
        if self._lmc is None:
            raise RuntimeError("GP must be trained before prediction. Call fit() first.")
        if variance_method not in ("love", "exact", "mean_only"):
            raise ValueError("variance_method must be one of 'love', 'exact', 'mean_only'")
        Xt = np.ascontiguousarray(X_test, np.float32)
        if Xt.ndim == 1 and self.dim == 1:
            Xt = Xt[:, None]
        _check_test_inputs(Xt, self.dim)
        T, n = self.T, self._X.shape[0]
        prov = self._lmc.providers[0]
        alpha = self._alpha.reshape(T, n).T
        Cs = prov.cross_matvec_host(Xt, alpha)  # [m, T]
        mean = (Cs @ self.task_covariance.T + self.mean_[None, :]).astype(np.float32)
        if variance_method == "mean_only":
            return _prediction_output(mean, None, return_var, return_std)
        from .gp import _DEFAULT_PREDICT_LANCZOS_RANK
        from .prediction import PredictionCache, exact_variance
        s2 = float(np.mean(self.noise_per_task))
        rank = lanczos_rank or max(_DEFAULT_PREDICT_LANCZOS_RANK,
                                   200 if self.kernel_resolved.has_ard() else 0)
        rank = min(rank, n)
        var = np.zeros((Xt.shape[0], T))
        try:
            for s in range(T):
                lam = float(self._Lambda[s])
                if lam <= 1e-8:
                    continue
                nz = s2 / lam
                prov.update_noise(nz)
                if variance_method == "love":
                    cache = PredictionCache(prov, np.zeros(n, np.float32), 0.0, rank)
                    _, v_s = cache.predict(Xt, return_var=True)
                    cache.destroy()
                else:
                    v_s, _ = exact_variance(prov, Xt, max_cg_iter=self.max_cg_iter,
                                            cg_tol=min(self.cg_tol, 1e-2), precond_rank=self.precond_rank)
                latent = np.maximum(v_s.astype(np.float64) - nz, 1e-10)
                var += (self._Q[:, s] ** 2 * lam)[None, :] * latent[:, None]
        finally:
            prov.update_noise(0.0)
        var = np.maximum(var, 0).astype(np.float32)
        return _prediction_output(mean, var, return_var, return_std)
