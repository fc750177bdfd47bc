"""SingleOutputGP: the reference's public single-output API on the B200 engine.

Mirrors mojogp/gp.py (SingleOutputGP 245-3949) for the matrix-free route:
  * fit(X, y, method="matrix_free") with the balanced/fast/accurate presets
    (gp.py:790-858), the matrix-free preconditioner defaults (1437-1457), the
    large-n 1-D/low-d RBF initial lengthscale tweak (1376-1408) and
    init_mean = mean(y) (1576-1578);
  * predict(X*, return_std / return_var, variance_method="love" | "mean_only")
    with the prediction solver config of gp.py:85-199 (alpha CG max(...,300)
    iterations at min(...,1e-3); LOVE rank max(max_tridiag, 100), 200 for ARD);
  * prepare_prediction_cache, log_marginal_likelihood (= -per-sample NLL,
    gp.py:3642-3646), get_params, save / load (JSON config + .npz arrays,
    gp.py:3648-3913).
Training and prediction run in the CUDA library (engine.py, prediction.py);
there is no CPU route. Multi-GPU: pass a distributed.Communicator as `comm`.
"""
from __future__ import annotations

import json
from dataclasses import dataclass
from pathlib import Path
from typing import Optional

import numpy as np

from . import engine, prediction
from .kernel import KernelNode, KernelType, make_ard_kernel
from .provider import Provider

# Saved-artifact schema of the reference (gp.py:76).
MODEL_SCHEMA_VERSION = 1


def _package_version() -> str:
    from . import __version__
    return __version__


def _artifact_base(path) -> str:
    path = str(path)
    if path.endswith(".json") or path.endswith(".npz"):
        path = path.rsplit(".", 1)[0]
    return path

_DEFAULT_PREDICT_LANCZOS_RANK = 100
_DEFAULT_ARD_PREDICT_LANCZOS_RANK = 200
_DEFAULT_PREDICT_MAX_CG_ITER = 300
_DEFAULT_PREDICT_CG_TOL = 1e-3


def _check_finite(name: str, a: np.ndarray) -> None:
    if not np.all(np.isfinite(a)):
        raise ValueError(f"{name} contains NaN or Inf values")


def _check_training_controls(max_iterations, learning_rate, initial_noise) -> None:
    """Optimiser argument checks with the reference's messages
    (SingleOutputGP.fit, gp.py:1270-1276; the multi-output fits check the same
    three, multi_output_gp.py:1555, 1613-1615, 4671-4675)."""
    if max_iterations <= 0:
        raise ValueError(f"max_iterations must be > 0, got {max_iterations}")
    if learning_rate <= 0:
        raise ValueError(f"learning_rate must be > 0, got {learning_rate}")
    if initial_noise <= 0:
        raise ValueError(f"initial_noise must be > 0, got {initial_noise}")


def _check_multi_output_data(X: np.ndarray, Y: np.ndarray) -> None:
    """Training data checks of the multi-output fits (multi_output_gp.py:1542-1553)."""
    if X.ndim != 2:
        raise ValueError(f"X must be 2D [n, d], got shape {X.shape}")
    if Y.ndim != 2:
        raise ValueError(f"Y must be 2D [n, T], got shape {Y.shape}")
    if X.shape[0] != Y.shape[0]:
        raise ValueError(f"X has {X.shape[0]} samples, Y has {Y.shape[0]} -- must match")
    _check_finite("X", X)
    _check_finite("Y", Y)


def _checked_observation_noise(noise, m: int, floor: float = 1e-6) -> np.ndarray:
    """Test-point observation noise for observed prediction (gp.py:2786-2798)."""
    if noise is None:
        raise ValueError("predict_observed()/predict(target='observed') requires "
                         "observation_noise for test points")
    obs = np.ascontiguousarray(noise, dtype=np.float32)
    if obs.shape != (m,):
        raise ValueError(f"observation_noise must have shape ({m},), got {obs.shape}")
    _check_finite("observation_noise", obs)
    if np.any(obs < floor):
        raise ValueError("observation_noise values must be >= noise_floor")
    return obs


def _check_test_inputs(Xt: np.ndarray, dim: int) -> None:
    """Prediction input checks (multi_output_gp.py:2565-2573)."""
    if Xt.ndim != 2:
        raise ValueError(f"X_test must be 2D [m, d], got shape {Xt.shape}")
    if Xt.shape[1] != dim:
        raise ValueError(f"X_test has {Xt.shape[1]} features, expected {dim}")
    _check_finite("X_test", Xt)


def _resolve_fit_route(method: str, n: int, dim: int, single_type, ard: bool,
                       learning_rate: float, default_params: bool, params: np.ndarray,
                       preconditioner, preconditioner_rank, use_preconditioner,
                       precond_rebuild_threshold) -> dict:
    """Training route and the defaults it implies (SingleOutputGP.fit,
    gp.py:1350-1468, continuous kernels). "auto" is the dense route up to 2000
    rows; the dense route (served here by the same matrix-free kernels) starts
    a 1-D RBF at lengthscale <= 0.5, picks greedy pivots for Matérn-3/2, no
    preconditioner for Linear, and rebuild threshold 0.1 for ARD stationary
    leaves; the matrix-free route starts a low-d isotropic RBF at <= 0.6 (n >=
    10000) and preconditions only that case (rank 256, n >= 5000) unless the
    caller asked. `single_type` is the KernelType of a one-leaf kernel, else
    None. Returns method, params, preconditioner, precond_rank (None = the
    preset's) and precond_rebuild_threshold."""
    if method in ("materialized", "mat"):
        route = "materialized"
    elif method == "auto":
        route = "materialized" if n <= 2000 else "matrix_free"
    else:
        route = "matrix_free"
    p = np.asarray(params, np.float32).copy()
    rbf = single_type == KernelType.RBF
    if default_params and route == "materialized" and learning_rate <= 0.05 and rbf and dim == 1 \
            and p.shape[0] >= 1:
        p[0] = min(float(p[0]), 0.5)
    if default_params and route == "matrix_free" and learning_rate <= 0.05 and rbf and not ard \
            and 1 < dim <= 8 and n >= 10000 and p.shape[0] >= 1:
        p[0] = min(float(p[0]), 0.6)
    explicit = (preconditioner is not None or preconditioner_rank is not None
                or use_preconditioner is not None)
    precond, rank = preconditioner, preconditioner_rank
    if precond is None and route == "materialized" and learning_rate <= 0.05 \
            and single_type == KernelType.MATERN32:
        precond = "greedy"
    if not explicit and route == "materialized" and single_type == KernelType.LINEAR:
        rank = 0
    if not explicit and route == "matrix_free":
        if rbf and not ard and 1 < dim <= 8 and n >= 5000:
            precond, rank = "greedy", 256
        else:
            rank = 0
    thr = precond_rebuild_threshold
    if thr is None and route == "materialized" and ard and single_type in (
            KernelType.RBF, KernelType.MATERN12, KernelType.MATERN32, KernelType.MATERN52,
            KernelType.RQ):
        thr = 0.1
    return {"method": route, "params": p, "preconditioner": precond, "precond_rank": rank,
            "precond_rebuild_threshold": thr}


def _prediction_lanczos_rank(rank_hint: Optional[int], is_ard: bool) -> int:
    """LOVE root rank: at least 100, at least 200 for ARD kernels
    (_prediction_lanczos_rank, gp.py:112-138, continuous kernels)."""
    rank = int(rank_hint) if rank_hint is not None else 0
    floor = _DEFAULT_PREDICT_LANCZOS_RANK
    if is_ard:
        floor = max(floor, _DEFAULT_ARD_PREDICT_LANCZOS_RANK)
    return max(rank, floor)


def _prediction_solver_config(train_info: Optional[dict], rank_hint: Optional[int], *,
                              is_ard: bool, max_cg_iterations: Optional[int] = None,
                              cg_tolerance: Optional[float] = None,
                              precond_rank: Optional[int] = None,
                              max_root_decomposition_size: Optional[int] = None) -> dict:
    """Prediction solver settings from the training settings and explicit
    overrides (_prediction_solver_config, gp.py:141-199, continuous kernels):
    CG iterations max(training, 300), tolerance min(training, 1e-3), the
    training preconditioner rank (10 when unknown), the LOVE rank above."""
    ti = train_info or {}
    pr = int(precond_rank if precond_rank is not None else ti.get("precond_rank", 10))
    rank = _prediction_lanczos_rank(rank_hint, is_ard)
    if max_root_decomposition_size is not None:
        rank = int(max_root_decomposition_size)
    it = int(ti.get("max_cg_iterations", ti.get("max_cg_iter", _DEFAULT_PREDICT_MAX_CG_ITER)))
    tol = float(ti.get("cg_tolerance", ti.get("cg_tol", _DEFAULT_PREDICT_CG_TOL)))
    return {
        "max_cg_iterations": int(max_cg_iterations if max_cg_iterations is not None
                                 else max(it, _DEFAULT_PREDICT_MAX_CG_ITER)),
        "cg_tolerance": float(cg_tolerance if cg_tolerance is not None
                              else min(tol, _DEFAULT_PREDICT_CG_TOL)),
        "precond_rank": pr,
        "max_root_decomposition_size": rank,
    }


@dataclass
class TrainingResult:
    params: np.ndarray
    noise: float
    mean: float
    nll: float
    iterations: int
    converged: bool
    lanczos_root: Optional[np.ndarray] = None
    lanczos_rank: int = 0
    nll_history: Optional[np.ndarray] = None
    cg_iterations_history: Optional[np.ndarray] = None
    iter_times_ms: Optional[np.ndarray] = None


@dataclass
class PredictionResult:
    mean: np.ndarray
    variance: np.ndarray
    std: np.ndarray


class SingleOutputGP:
    """Exact GP with a composable kernel, trained matrix-free on B200."""

    _PRESETS = {
        "fast": {"max_cg_iter": 50, "cg_tol": 5e-2, "num_probes": 5, "max_tridiag_iter": 15,
                 "precond_rank": 50, "precond_rebuild_threshold": 0.75, "precond": "greedy"},
        "balanced": {"max_cg_iter": 100, "cg_tol": 1e-2, "num_probes": 10, "max_tridiag_iter": 30,
                     "precond_rank": 100, "precond_rebuild_threshold": 0.5, "precond": "greedy"},
        "accurate": {"max_cg_iter": 200, "cg_tol": 1e-3, "num_probes": 20, "max_tridiag_iter": 60,
                     "precond_rank": 200, "precond_rebuild_threshold": 0.25, "precond": "greedy"},
    }

    def __init__(self, kernel: KernelNode, *, init_mean: Optional[float] = None,
                 verbose: bool = False, device: int = 0):
        if not isinstance(kernel, KernelNode):
            raise TypeError(
                f"kernel must be a KernelNode instance (e.g. RBF(), Matern52()), got "
                f"{type(kernel).__name__}")
        self.kernel_spec = kernel
        self.kernel: Optional[KernelNode] = None
        self.ard = kernel.has_ard()
        self.verbose = verbose
        self.device = device
        self._init_mean = init_mean
        self._X_train = None
        self._y_train = None
        self._obs_noise = None
        self._provider: Optional[Provider] = None
        self._training_result: Optional[TrainingResult] = None
        self._train_info: dict = {}
        self._cache = None
        self._cache_key = None
        self._comm = None
        self.dim = None

    # ----------------------------------------------------------------- helpers
    @staticmethod
    def _resolve_cg_params(preset=None, **over) -> dict:
        base = dict(SingleOutputGP._PRESETS[preset or "balanced"])
        for k, v in over.items():
            if v is not None:
                base[k] = v
        return base

    def _resolved_kernel(self, dim: int) -> KernelNode:
        return make_ard_kernel(self.kernel_spec, dim) if self.ard else self.kernel_spec.resolve_ard(dim)

    def _single_type(self, kt: KernelType) -> bool:
        k = self.kernel_spec
        return k.is_leaf() and k.kernel_type == kt

    @property
    def _is_trained(self) -> bool:
        return self._training_result is not None

    # -------------------------------------------------------------------- fit
    def fit(self, X, y, max_iterations: int = 100, learning_rate: float = 0.01,
            initial_noise: float = 0.1, initial_params: Optional[np.ndarray] = None,
            method: str = "auto", enable_early_stopping: bool = False,
            early_stop_patience: int = 10, early_stop_tol: float = 1e-4,
            verbose: Optional[bool] = None, preset: Optional[str] = None,
            max_cg_iterations: Optional[int] = None, cg_tolerance: Optional[float] = None,
            num_probes: Optional[int] = None, max_tridiag_iterations: Optional[int] = None,
            preconditioner_rank: Optional[int] = None,
            precond_rebuild_threshold: Optional[float] = None,
            preconditioner: Optional[str] = None, use_preconditioner: Optional[bool] = None,
            lr_schedule: str = "constant", prepare_prediction_cache: bool = False,
            prediction_cache_rank: Optional[int] = None,
            observation_noise: Optional[np.ndarray] = None, learn_noise: bool = True,
            comm=None) -> TrainingResult:
        """Train hyperparameters by BBMM (mBCG + SLQ) with Adam on the GPU."""
        X = np.ascontiguousarray(X, dtype=np.float32)
        y = np.ascontiguousarray(y, dtype=np.float32)
        # Data, then optimiser checks, with the reference's messages (gp.py:995-1004, 1266-1284).
        if X.ndim != 2:
            raise ValueError(f"X must be 2D, got shape {X.shape}")
        if y.ndim != 1:
            raise ValueError(f"y must be 1D, got shape {y.shape}")
        if X.shape[0] != y.shape[0]:
            raise ValueError(f"X has {X.shape[0]} samples, y has {y.shape[0]}")
        if X.shape[0] == 0:
            raise ValueError("cannot fit on an empty dataset")
        _check_finite("X", X)
        _check_finite("y", y)
        if preset is not None and preset not in self._PRESETS:
            raise ValueError(f"Unknown preset '{preset}'. Must be one of: {list(self._PRESETS.keys())}")
        _check_training_controls(max_iterations, learning_rate, initial_noise)
        if early_stop_patience < 0:
            raise ValueError(f"early_stop_patience must be >= 0, got {early_stop_patience}")
        if early_stop_tol < 0:
            raise ValueError(f"early_stop_tol must be >= 0, got {early_stop_tol}")
        if prediction_cache_rank is not None and prediction_cache_rank <= 0:
            raise ValueError("prediction_cache_rank must be positive or None")
        if method not in ("auto", "matrix_free", "mf", "materialized", "mat"):
            raise ValueError(f"method={method!r}: expected 'auto', 'matrix_free' or 'materialized'")
        # The materialized route (dense K + GEMM for n <= ~4e4) is served by the
        # matrix-free tile kernels: re-evaluating K on the tensor cores costs less
        # than streaming a stored K from HBM at t = 16 (fn_ptr_module.py:363-421).
        if lr_schedule not in ("constant", "cosine"):
            raise ValueError(f"lr_schedule must be 'cosine' or 'constant', got '{lr_schedule}'")
        n, dim = X.shape
        self.dim = dim
        self._comm = comm
        self.kernel = self._resolved_kernel(dim)
        P = self.kernel.num_params()
        default_params = initial_params is None
        params = (self.kernel.get_initial_params() if default_params
                  else np.asarray(initial_params, np.float32).ravel())
        if params.shape[0] != P:
            raise ValueError(f"initial_params must have {P} entries, got {params.shape[0]}")
        k = self.kernel_spec
        route = _resolve_fit_route(method, n, dim, k.kernel_type if k.is_leaf() else None,
                                   self.ard, learning_rate, default_params, params, preconditioner,
                                   preconditioner_rank, use_preconditioner,
                                   precond_rebuild_threshold)
        self._training_method = route["method"]
        params = route["params"]
        preconditioner, rank = route["preconditioner"], route["precond_rank"]
        precond_rebuild_threshold = route["precond_rebuild_threshold"]
        if preconditioner not in (None, "greedy"):
            raise NotImplementedError(
                f"preconditioner={preconditioner!r}: only the greedy pivoted Cholesky is built")
        cg = self._resolve_cg_params(preset, max_cg_iter=max_cg_iterations, cg_tol=cg_tolerance,
                                     num_probes=num_probes,
                                     max_tridiag_iter=max_tridiag_iterations,
                                     precond_rank=rank,
                                     precond_rebuild_threshold=precond_rebuild_threshold)
        use_p = bool(use_preconditioner) if use_preconditioner is not None else cg["precond_rank"] > 0
        if observation_noise is not None:
            use_p = False  # the Woodbury preconditioner assumes scalar noise
        init_mean = float(np.mean(y)) if self._init_mean is None else float(self._init_mean)
        self._destroy()
        self._X_train, self._y_train = X, y
        self._obs_noise = None if observation_noise is None else np.asarray(observation_noise, np.float32)
        self._provider = Provider(X, self.kernel, params, initial_noise, device=self.device,
                                  noise_vector=self._obs_noise)
        res = engine.train(
            self._provider, y, max_iterations=max_iterations, learning_rate=learning_rate,
            num_probes=cg["num_probes"], max_cg_iter=cg["max_cg_iter"], cg_tol=cg["cg_tol"],
            precond_rank=cg["precond_rank"] if use_p else 0,
            max_tridiag_iter=cg["max_tridiag_iter"],
            precond_rebuild_threshold=cg["precond_rebuild_threshold"],
            use_cosine_lr=lr_schedule == "cosine", use_preconditioner=use_p,
            learn_noise=learn_noise, init_mean=init_mean,
            enable_early_stopping=enable_early_stopping, early_stop_patience=early_stop_patience,
            early_stop_tol=early_stop_tol,
            verbose=self.verbose if verbose is None else verbose,
            trainable_mask=self.kernel.engine_trainable_mask(), comm=comm)
        self._train_info = {"max_cg_iterations": cg["max_cg_iter"], "cg_tolerance": cg["cg_tol"],
                            "max_tridiag_iter": cg["max_tridiag_iter"],
                            "precond_rank": res["precond_rank"],
                            "precond_build_count": res["precond_build_count"],
                            "precond_build_time_ms": res["precond_build_time_ms"],
                            "tile_kernels": res["tile_kernels"]}
        self._training_result = TrainingResult(
            params=res["params"], noise=res["noise"], mean=res["mean"], nll=res["final_nll"],
            iterations=res["iterations"], converged=res["converged"],
            lanczos_rank=cg["max_tridiag_iter"], nll_history=res["nll_history"],
            cg_iterations_history=res["cg_iterations_history"],
            iter_times_ms=res["iter_times_ms"])
        if prepare_prediction_cache:
            self.prepare_prediction_cache(max_root_decomposition_size=prediction_cache_rank)
        return self._training_result

    # ---------------------------------------------------------------- predict
    def _solver_config(self, max_cg_iterations=None, cg_tolerance=None,
                       max_root_decomposition_size=None, precond_rank=None) -> dict:
        cfg = _prediction_solver_config(
            self._train_info, int(self._training_result.lanczos_rank), is_ard=self.ard,
            max_cg_iterations=max_cg_iterations, cg_tolerance=cg_tolerance,
            precond_rank=precond_rank, max_root_decomposition_size=max_root_decomposition_size)
        # A root cannot have more Lanczos vectors than training rows.
        cfg["max_root_decomposition_size"] = min(cfg["max_root_decomposition_size"],
                                                 self._X_train.shape[0])
        return cfg

    def prepare_prediction_cache(self, variance_method: str = "love",
                                 max_root_decomposition_size: Optional[int] = None,
                                 max_cg_iterations: Optional[int] = None,
                                 cg_tolerance: Optional[float] = None):
        if not self._is_trained:
            raise RuntimeError("GP must be trained first.")
        cfg = self._solver_config(max_cg_iterations, cg_tolerance, max_root_decomposition_size)
        rank = cfg["max_root_decomposition_size"] if variance_method == "love" else 0
        key = (cfg["max_cg_iterations"], cfg["cg_tolerance"], rank)
        if self._cache is not None and self._cache_key == key:
            return self._cache
        tr = self._training_result
        alpha, _ = prediction.compute_alpha(self._provider, self._y_train - tr.mean,
                                            cfg["max_cg_iterations"], cfg["cg_tolerance"],
                                            comm=self._comm)
        root = tr.lanczos_root if (tr.lanczos_root is not None and rank > 0 and
                                   tr.lanczos_root.shape == (rank, self._X_train.shape[0])) else None
        self._cache = prediction.PredictionCache(self._provider, alpha, tr.mean, rank, root=root,
                                                 comm=self._comm)
        if rank > 0 and root is None:
            tr.lanczos_root = self._cache.root()
        self._cache_key = key
        self._alpha = alpha
        return self._cache

    def predict(self, X_test, return_std: bool = False, return_var: bool = False,
                variance_method: str = "love", max_cg_iterations: Optional[int] = None,
                cg_tolerance: Optional[float] = None,
                max_root_decomposition_size: Optional[int] = None,
                preconditioner_rank: Optional[int] = None,
                exact_prediction_block_cols: Optional[int] = None, target: str = "latent",
                observation_noise: Optional[np.ndarray] = None):
        """Predictive mean and variance / std: LOVE (variance_method="love"),
        CG-exact ("exact") or none ("mean_only"). As the reference's engine does
        (jit_prediction.mojo:2048-2051), the variance includes the learned noise;
        target="observed" adds the given test-point `observation_noise` [m] on
        top (predict / _add_observation_noise_to_prediction, gp.py:2446-2809).
        Returns (mean, var) with return_var, (mean, std) with return_std,
        otherwise a PredictionResult."""
        if not self._is_trained:
            raise RuntimeError("GP must be trained before prediction. Call fit() first.")
        if return_var and return_std:
            raise ValueError("Only one of return_var or return_std may be True.")
        if variance_method not in ("love", "exact", "mean_only"):
            raise ValueError("variance_method must be one of 'love', 'exact', 'mean_only'")
        if target not in ("latent", "observed"):
            raise ValueError("target must be 'latent' or 'observed'")
        if exact_prediction_block_cols is not None and exact_prediction_block_cols <= 0:
            raise ValueError("exact_prediction_block_cols must be positive or None")
        Xt = np.ascontiguousarray(X_test, dtype=np.float32)
        if Xt.ndim == 1 and self.dim == 1:
            Xt = Xt[:, None]
        _check_test_inputs(Xt, self.dim)
        want_var = variance_method == "love"
        cache = self.prepare_prediction_cache("love" if want_var else "mean_only",
                                              max_root_decomposition_size, max_cg_iterations,
                                              cg_tolerance)
        if self._comm is not None and self._comm.world > 1:
            mean, var = cache.predict_sharded(Xt, self._comm, return_var=want_var)
        else:
            mean, var = cache.predict(Xt, return_var=want_var)
        if variance_method == "exact":
            # The exact route's solver settings (_prediction_solver_config):
            # iterations max(training, 300), tolerance min(training, 1e-3), the
            # training preconditioner rank.
            from .prediction import exact_variance
            cfg = self._solver_config(max_cg_iterations, cg_tolerance, None, preconditioner_rank)
            var, _ = exact_variance(
                self._provider, Xt, max_cg_iter=cfg["max_cg_iterations"],
                cg_tol=cfg["cg_tolerance"], precond_rank=cfg["precond_rank"],
                block_cols=exact_prediction_block_cols or 0, comm=self._comm)
        if var is None:
            var = np.zeros_like(mean)
        if target == "observed":
            var = var + _checked_observation_noise(observation_noise, Xt.shape[0])
        std = np.sqrt(np.maximum(var, 0))
        if return_var:
            return mean, var
        if return_std:
            return mean, std
        return PredictionResult(mean=mean, variance=var, std=std)

    def predict_latent(self, X, **kwargs):
        """p(f_test | y_train) (predict_latent, gp.py:2676-2679)."""
        kwargs.pop("target", None)
        return self.predict(X, target="latent", **kwargs)

    def predict_observed(self, X, observation_noise: Optional[np.ndarray] = None, **kwargs):
        """p(y_test | y_train) with explicit test-point noise (predict_observed,
        gp.py:2681-2700): the training noise is never reused for new points."""
        kwargs.pop("target", None)
        return self.predict(X, target="observed", observation_noise=observation_noise, **kwargs)

    def score(self, X_test, y_test) -> float:
        """R^2 of the predictive mean (score, gp.py:3059-3070)."""
        if not self._is_trained:
            raise RuntimeError("Model must be trained before scoring")
        y_test = np.asarray(y_test, dtype=np.float32)
        mean, _ = self.predict(np.asarray(X_test, dtype=np.float32), return_std=True)
        ss_res = float(np.sum((y_test - mean) ** 2))
        ss_tot = float(np.sum((y_test - np.mean(y_test)) ** 2))
        return 0.0 if ss_tot == 0 else 1.0 - ss_res / ss_tot

    # Reference read-only members (gp.py:740-779).
    @property
    def num_params(self) -> int:
        return (self.kernel or self.kernel_spec).num_params()

    @property
    def param_names(self) -> list:
        return (self.kernel or self.kernel_spec).get_param_names()

    @property
    def is_trained(self) -> bool:
        return self._is_trained

    @property
    def training_result(self) -> Optional[TrainingResult]:
        return self._training_result

    @property
    def nll_history(self) -> Optional[np.ndarray]:
        return None if self._training_result is None else self._training_result.nll_history

    @property
    def backend_train_info(self) -> Optional[dict]:
        return dict(self._train_info) if self._train_info else None

    # ---------------------------------------------------------------- queries
    def log_marginal_likelihood(self) -> float:
        if not self._is_trained:
            raise RuntimeError("GP must be trained first.")
        return -float(self._training_result.nll)

    def get_learned_params(self) -> dict:
        """Learned kernel parameters by name, then noise and mean
        (get_learned_params, gp.py:3072-3099, homoskedastic noise)."""
        if not self._is_trained:
            raise RuntimeError("Model must be trained before getting params")
        tr = self._training_result
        out = dict(zip(self.kernel.get_param_names(), map(float, tr.params)))
        out["noise"] = float(tr.noise)
        out["mean"] = float(tr.mean)
        return out

    def get_params(self) -> dict:
        return self.get_learned_params()

    @property
    def noise(self) -> float:
        return float(self._training_result.noise)

    @property
    def mean(self) -> float:
        return float(self._training_result.mean)

    # -------------------------------------------------------------- persist
    def _artifact_config(self) -> dict:
        """The reference's `{path}_config.json` content (gp.py:3661-3707) for
        this continuous-kernel model; keys the reference's load() reads
        (gp.py:3735-3876) carry the same meaning here."""
        tr = self._training_result
        return {
            "schema_version": MODEL_SCHEMA_VERSION,
            "mojogp_version": f"mojogp_b200 {_package_version()}",
            "wrapper": "SingleOutputGP",
            "dim": int(self.dim),
            "ard": bool(self.ard),
            "verbose": bool(self.verbose),
            "cat_dims": {},
            "cat_kernel": "ehh",
            "kernel_tree": self.kernel_spec.to_dict(),
            "is_mixed": False,
            "training_method": self._training_method,
            "engine_mean": None,
            "backend_train_info": self._train_info or None,
            "cached_love_method": None,
            "noise_mode": "scalar" if self._obs_noise is None else "fixed_vector",
            "noise_floor": 1e-6,
            "noise_regularization": 0.0,
            "noise_function": None,
            "provider_noise_mode_int": None if self._obs_noise is None else 1,
            "has_observation_noise_train": self._obs_noise is not None,
            "has_observation_noise_fn": False,
            "has_noise_group_train": False,
            "has_group_noise": False,
            "result_type": "TrainingResult",
            "noise": float(tr.noise),
            "mean": float(tr.mean),
            "nll": float(tr.nll),
            "iterations": int(tr.iterations),
            "converged": bool(tr.converged),
            "lanczos_rank": int(tr.lanczos_rank),
        }

    def save(self, path: str) -> None:
        """Save the trained model in the reference's artifact layout
        (gp.py:3648-3723): `{path}_config.json` and `{path}_arrays.npz` with
        X_train, y_train, params (and observation_noise_train). A cached LOVE
        root is stored as the extra array `lanczos_root`, which the
        reference's load ignores. A trailing .json / .npz on `path` is
        dropped, as in the reference."""
        if not self._is_trained:
            raise RuntimeError("GP must be trained before saving.")
        base = _artifact_base(path)
        tr = self._training_result
        with open(f"{base}_config.json", "w") as f:
            json.dump(self._artifact_config(), f, indent=2)
        arrays = {"X_train": self._X_train, "y_train": self._y_train,
                  "params": np.asarray(tr.params, np.float32)}
        if self._obs_noise is not None:
            arrays["observation_noise_train"] = self._obs_noise
        if tr.lanczos_root is not None:
            arrays["lanczos_root"] = tr.lanczos_root
        np.savez(f"{base}_arrays.npz", **arrays)

    @staticmethod
    def read_artifact(path: str):
        """Read and check a saved SingleOutputGP artifact (the reference's
        checks and messages, gp.py:3735-3770); returns (config, arrays).
        Needs no GPU."""
        base = _artifact_base(path)
        with open(f"{base}_config.json", "r") as f:
            config = json.load(f)
        wrapper = config.get("wrapper")
        if wrapper != "SingleOutputGP":
            raise ValueError(
                "Saved model is not a SingleOutputGP artifact. "
                f"Expected wrapper='SingleOutputGP', got {wrapper!r}.")
        schema_version = int(config.get("schema_version", 0))
        if schema_version != MODEL_SCHEMA_VERSION:
            raise ValueError(
                f"Unsupported SingleOutputGP schema_version={schema_version}; "
                f"expected {MODEL_SCHEMA_VERSION}.")
        if "kernel_tree" not in config:
            raise ValueError("SingleOutputGP artifact is missing required kernel_tree.")
        if config.get("is_mixed") or config.get("cat_dims"):
            raise NotImplementedError("mixed / categorical kernels are not built")
        if config.get("result_type", "TrainingResult") != "TrainingResult":
            raise NotImplementedError(f"result_type {config.get('result_type')!r} is not built")
        with np.load(f"{base}_arrays.npz", allow_pickle=False) as npz:
            arrays = {k: npz[k] for k in npz.files}
        return config, arrays

    @classmethod
    def load(cls, path: str, kernel: Optional[KernelNode] = None,
             device: int = 0) -> "SingleOutputGP":
        """Load an artifact written by save() here or by the reference's
        SingleOutputGP.save (gp.py:3725-3910): the kernel comes from
        `kernel_tree` unless given, the trained state from the config and
        arrays; the provider is created on `device`."""
        config, arrays = cls.read_artifact(path)
        if kernel is None:
            kernel = KernelNode.from_dict(config["kernel_tree"])
        gp = cls(kernel, init_mean=config.get("init_mean"), verbose=config.get("verbose", False),
                 device=device)
        X = np.ascontiguousarray(arrays["X_train"], dtype=np.float32)
        y = np.ascontiguousarray(arrays["y_train"], dtype=np.float32)
        gp.dim = X.shape[1]
        gp.kernel = gp._resolved_kernel(gp.dim)
        gp._X_train, gp._y_train = X, y
        gp._obs_noise = (np.ascontiguousarray(arrays["observation_noise_train"], np.float32)
                         if "observation_noise_train" in arrays else None)
        gp._training_method = config.get("training_method")
        gp._train_info = dict(config.get("backend_train_info") or {})
        params = np.ascontiguousarray(arrays["params"], dtype=np.float32)
        if params.shape[0] != gp.kernel.num_params():
            raise ValueError(f"saved params have {params.shape[0]} entries, the kernel needs "
                             f"{gp.kernel.num_params()}")
        gp._training_result = TrainingResult(
            params=params, noise=config["noise"], mean=config.get("mean", 0.0),
            nll=config["nll"], iterations=config["iterations"], converged=config["converged"],
            lanczos_root=arrays.get("lanczos_root"), lanczos_rank=config["lanczos_rank"])
        gp._provider = Provider(X, gp.kernel, params, float(config["noise"]), device=device,
                                noise_vector=gp._obs_noise)
        return gp

    def _destroy(self) -> None:
        if self._cache is not None:
            self._cache.destroy()
        self._cache = None
        self._cache_key = None
        if self._provider is not None:
            self._provider.destroy()
        self._provider = None
        self._training_result = None

    def __del__(self):
        try:
            self._destroy()
        except Exception:
            pass


def fit_gp(X: np.ndarray, y: np.ndarray, kernel: Optional[KernelNode] = None,
           **kwargs) -> SingleOutputGP:
    """Create and fit a SingleOutputGP in one call (fit_gp, gp.py:3928-3949);
    the kernel defaults to RBF and the keyword arguments go to fit()."""
    from .kernel import Kernel
    gp = SingleOutputGP(kernel if kernel is not None else Kernel.rbf())
    gp.fit(X, y, **kwargs)
    return gp
