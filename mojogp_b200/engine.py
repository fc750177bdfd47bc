"""Engine protocol over the C ABI: train / bbmm / predict.

Keeps the reference engine's call shapes and result-dict keys
(mojogp/kernels/jit/jit_engine_bindings.mojo:123-432 train, 944-1234 predict,
636-942 prediction cache) so the orchestration in gp.py reads like the
reference's gp.py:1608-2047.
"""
from __future__ import annotations

import ctypes as C
from typing import Optional

import numpy as np

from . import _lib
from .provider import Provider


class TrainOptions(C.Structure):
    _fields_ = [
        ("max_iterations", C.c_int32),
        ("learning_rate", C.c_float),
        ("num_probes", C.c_int32),
        ("max_cg_iter", C.c_int32),
        ("cg_tol", C.c_float),
        ("precond_rank", C.c_int32),
        ("max_tridiag_iter", C.c_int32),
        ("precond_rebuild_threshold", C.c_float),
        ("use_cosine_lr", C.c_int32),
        ("use_preconditioner", C.c_int32),
        ("learn_noise", C.c_int32),
        ("init_mean", C.c_float),
        ("enable_early_stopping", C.c_int32),
        ("early_stop_patience", C.c_int32),
        ("early_stop_tol", C.c_float),
        ("verbose", C.c_int32),
        ("trainable_mask", C.c_void_p),
    ]


class TrainResult(C.Structure):
    _fields_ = [
        ("final_nll", C.c_float),
        ("noise", C.c_float),
        ("mean", C.c_float),
        ("iterations", C.c_int32),
        ("converged", C.c_int32),
        ("params", C.c_void_p),
        ("nll_history", C.c_void_p),
        ("iter_times_ms", C.c_void_p),
        ("cg_iterations", C.c_void_p),
        ("alpha", C.c_void_p),
        ("alpha_valid", C.c_int32),
        ("precond_build_count", C.c_int32),
        ("precond_build_ms", C.c_double),
        ("precond_rank", C.c_int32),
        ("tile_layouts", C.c_void_p),
    ]


def _p(a: np.ndarray) -> C.c_void_p:
    return C.c_void_p(a.ctypes.data)


def train(provider: Provider, y: np.ndarray, *, max_iterations: int = 100,
          learning_rate: float = 0.01, num_probes: int = 10, max_cg_iter: int = 100,
          cg_tol: float = 1e-2, precond_rank: int = 100, max_tridiag_iter: int = 30,
          precond_rebuild_threshold: float = 0.5, use_cosine_lr: bool = False,
          use_preconditioner: bool = True, learn_noise: bool = True, init_mean: float = 0.0,
          enable_early_stopping: bool = False, early_stop_patience: int = 10,
          early_stop_tol: float = 1e-4, verbose: bool = False,
          trainable_mask: Optional[np.ndarray] = None, comm=None) -> dict:
    """Run the training loop on the device; returns the reference's result keys."""
    y = np.ascontiguousarray(y, dtype=np.float32).ravel()
    if y.shape[0] != provider.n:
        raise ValueError(f"y has {y.shape[0]} rows, provider has {provider.n}")
    P = provider.num_params
    mask = None
    if trainable_mask is not None:
        mask = np.ascontiguousarray(trainable_mask, dtype=np.uint8)
    opt = TrainOptions(max_iterations, learning_rate, num_probes, max_cg_iter, cg_tol,
                       precond_rank, max_tridiag_iter, precond_rebuild_threshold,
                       int(use_cosine_lr), int(use_preconditioner), int(learn_noise), init_mean,
                       int(enable_early_stopping), early_stop_patience, early_stop_tol,
                       int(verbose), _p(mask) if mask is not None else None)
    params = np.zeros(P, np.float32)
    nll_hist = np.full(max(max_iterations, 1), np.nan, np.float32)
    times = np.zeros(max(max_iterations, 1), np.float64)
    cg_it = np.zeros(max(max_iterations, 1), np.int32)
    alpha = np.zeros(provider.n, np.float32)
    res = TrainResult()
    res.params = _p(params).value
    res.nll_history = _p(nll_hist).value
    res.iter_times_ms = _p(times).value
    res.cg_iterations = _p(cg_it).value
    res.alpha = _p(alpha).value
    layouts = np.full(max(max_iterations, 1), -1, np.int32)
    res.tile_layouts = _p(layouts).value
    _lib.call("gpb_train", provider.h, C.c_void_p(comm.handle) if comm else None, _p(y),
              provider.n, C.byref(opt), C.byref(res))
    it = int(res.iterations)
    provider._params = params.copy()
    provider._noise = float(res.noise)
    return {
        "final_nll": float(res.final_nll),
        "noise": float(res.noise),
        "mean": float(res.mean),
        "iterations": it,
        "converged": bool(res.converged),
        "params": params,
        "iter_times_ms": times[:it].copy(),
        "nll_history": nll_hist[:it].copy(),
        "cg_iterations_history": cg_it[:it].copy(),
        "cached_alpha": alpha if res.alpha_valid else None,
        "precond_build_count": int(res.precond_build_count),
        "precond_build_time_ms": float(res.precond_build_ms),
        "precond_rank": int(res.precond_rank),
        "tile_kernels": [Provider.LAYOUTS.get(int(v), str(int(v))) for v in layouts[:it]],
    }


def train_binding(info, y, params, noise, max_iterations=100, learning_rate=0.01, num_probes=10,
                  max_cg_iter=100, cg_tol=1e-2, precond_rank=10, verbose=False,
                  use_cosine_lr=True, use_preconditioner=True, max_tridiag_iter=30,
                  precond_rebuild_threshold=0.5, precond_method=0, init_mean=0.0,
                  enable_early_stopping=False, early_stop_patience=10, early_stop_tol=1e-4,
                  learn_noise=True, noise_floor=1e-6, noise_regularization=0.01,
                  progress_callback=None, progress_interval=1, *, trainable_mask=None,
                  comm=None) -> dict:
    """The reference engine's `train` with its positional argument order
    (train_python, jit_engine_bindings.mojo:123-247) and result keys (336-432),
    over `train` above: the provider takes `params` and `noise` first. Only the
    greedy pivoted Cholesky (precond_method 0) and the homoskedastic learned
    noise with the reference's default floor / regularisation are built; a
    progress callback is not supported (training runs as one device call)."""
    if int(precond_method) != 0:
        raise NotImplementedError(
            f"precond_method={precond_method}: only the greedy pivoted Cholesky (0) is built")
    if float(noise_floor) != 1e-6 or float(noise_regularization) != 0.01:
        raise NotImplementedError("noise_floor / noise_regularization other than the defaults "
                                  "belong to the learned-noise models, which are not built")
    if progress_callback is not None:
        raise NotImplementedError("progress callbacks are not supported")
    prov = info["provider"] if isinstance(info, dict) else info
    prov.update_params(np.asarray(params, dtype=np.float32))
    prov.update_noise(float(noise))
    res = train(prov, y, max_iterations=int(max_iterations), learning_rate=float(learning_rate),
                num_probes=int(num_probes), max_cg_iter=int(max_cg_iter), cg_tol=float(cg_tol),
                precond_rank=int(precond_rank), max_tridiag_iter=int(max_tridiag_iter),
                precond_rebuild_threshold=float(precond_rebuild_threshold),
                use_cosine_lr=bool(use_cosine_lr), use_preconditioner=bool(use_preconditioner),
                learn_noise=bool(learn_noise), init_mean=float(init_mean),
                enable_early_stopping=bool(enable_early_stopping),
                early_stop_patience=int(early_stop_patience), early_stop_tol=float(early_stop_tol),
                verbose=bool(verbose), trainable_mask=trainable_mask, comm=comm)
    mode = int(info.get("materialization_mode", 0)) if isinstance(info, dict) else 0
    res.update({
        "training_route": "materialized" if mode == 1 else "matrix_free",
        "materialization_mode": mode,
        "is_ard": bool(info.get("is_ard", False)) if isinstance(info, dict) else False,
        "noise_mode": "scalar",
        "learn_noise": bool(learn_noise),
        "noise_floor": float(noise_floor),
        "noise_regularization": float(noise_regularization),
        "use_preconditioner": bool(use_preconditioner),
        "precond_method": int(precond_method),
        "max_tridiag_iter": int(max_tridiag_iter),
        "precond_rebuild_threshold": float(precond_rebuild_threshold),
        "enable_early_stopping": bool(enable_early_stopping),
        "early_stop_patience": int(early_stop_patience),
        "early_stop_tol": float(early_stop_tol),
        "precond_rank": int(precond_rank),
        "actual_precond_rank": int(res["precond_rank"]),
        "precond_rebuild_count": max(0, int(res["precond_build_count"]) - 1),
        "precond_build_total_ms": float(res["precond_build_time_ms"]),
    })
    return res


def bbmm(provider: Provider, y_centered: np.ndarray, *, num_probes: int = 10,
         max_cg_iter: int = 100, max_tridiag_iter: int = 30, cg_tol: float = 1e-2,
         precond_rank: int = 0, iteration: int = 0, comm=None) -> dict:
    """One NLL + gradient evaluation at the provider's parameters."""
    y = np.ascontiguousarray(y_centered, dtype=np.float32).ravel()
    nll = C.c_double()
    grads = np.zeros(provider.num_params + 1, np.float64)
    ld, iq = C.c_double(), C.c_double()
    it = C.c_int32()
    _lib.call("gpb_bbmm", provider.h, C.c_void_p(comm.handle) if comm else None, _p(y),
              provider.n, num_probes, max_cg_iter, max_tridiag_iter, float(cg_tol), precond_rank,
              iteration, C.byref(nll), _p(grads), C.byref(ld), C.byref(iq), C.byref(it))
    return {"nll": nll.value, "grads": grads, "logdet": ld.value, "inv_quad": iq.value,
            "cg_iters": it.value}


def precond_pivots(provider: Provider, rank: int, comm=None) -> dict:
    """Greedy pivoted-Cholesky pivots at the provider's parameters, in pick
    order, with the residual diagonal each was picked at (the build that
    gpb_bbmm / gpb_train run; pivoted_cholesky.mojo:500-609, 772-1050)."""
    piv = np.zeros(max(int(rank), 1), np.int64)
    val = np.zeros(max(int(rank), 1), np.float32)
    got = C.c_int32()
    _lib.call("gpb_precond_pivots", provider.h, C.c_void_p(comm.handle) if comm else None,
              int(rank), _p(piv), _p(val), C.byref(got))
    return {"pivots": piv[:got.value].copy(), "values": val[:got.value].copy()}


PREDICT_MEAN_ONLY, PREDICT_LOVE, PREDICT_EXACT = 0, 1, 2
_DEFAULT_LOVE_RANK, _DEFAULT_ARD_LOVE_RANK = 100, 200
_CACHES: dict = {}  # live prediction caches by handle (prepare / predict_with_cache / destroy)


def _provider_of(info):
    return info["provider"] if isinstance(info, dict) else info


def _check_variance_method(variance_method) -> None:
    if variance_method not in (PREDICT_MEAN_ONLY, PREDICT_LOVE, PREDICT_EXACT):
        raise ValueError(f"variance_method must be 0, 1 or 2, got {variance_method}")


def _build_cache(info, y, params, final_noise, final_mean, variance_method, max_cg_iter, cg_tol,
                 lanczos_rank, provider_state_current, cached_alpha, cached_love_root, comm):
    """Provider update, alpha (CG or cached) and the LOVE root (Lanczos or
    cached) in a device prediction cache; returns (cache, alpha, facts)."""
    import time

    from . import prediction

    _check_variance_method(variance_method)
    prov = _provider_of(info)
    n = prov.n
    if not provider_state_current:
        prov.update_params(np.asarray(params, dtype=np.float32))
        prov.update_noise(float(final_noise))
    t0 = time.perf_counter()
    alpha_cache_used = cached_alpha is not None
    if alpha_cache_used:
        alpha = np.ascontiguousarray(cached_alpha, dtype=np.float32).ravel()
        if alpha.shape[0] != n:
            raise ValueError(f"cached alpha has {alpha.shape[0]} values, expected {n}")
    else:
        yc = np.ascontiguousarray(y, dtype=np.float32).ravel() - np.float32(final_mean)
        alpha, _ = prediction.compute_alpha(prov, yc, max_cg_iter, cg_tol, comm=comm)
    alpha_s = time.perf_counter() - t0
    rank, root, root_cached = 0, None, False
    if variance_method == PREDICT_LOVE:
        # _resolve_exact_predict_lanczos_rank (jit_engine_binding_helpers.mojo:23-45)
        is_ard = bool(info.get("is_ard", False)) if isinstance(info, dict) else False
        rank = lanczos_rank if lanczos_rank > 0 else (
            _DEFAULT_ARD_LOVE_RANK if is_ard else _DEFAULT_LOVE_RANK)
        rank = min(rank, n)
        if cached_love_root is not None:
            r = np.ascontiguousarray(cached_love_root, dtype=np.float32).ravel()
            if r.shape[0] == n * rank:
                root, root_cached = r.reshape(rank, n), True
    t1 = time.perf_counter()
    cache = prediction.PredictionCache(prov, alpha, float(final_mean), rank, root=root, comm=comm)
    root_s = time.perf_counter() - t1 if (rank > 0 and not root_cached) else 0.0
    facts = {"alpha_time_s": alpha_s, "love_root_time_s": root_s,
             "alpha_cache_used": alpha_cache_used, "love_root_cache_used": root_cached,
             "rank": rank}
    return cache, alpha, facts


def _predict_from_cache(info, cache, x_test, params, final_noise, variance_method, max_cg_iter,
                        cg_tol, precond_rank, provider_state_current, exact_block_cols, comm):
    import time

    from . import prediction

    _check_variance_method(variance_method)
    prov = _provider_of(info)
    if not provider_state_current:
        prov.update_params(np.asarray(params, dtype=np.float32))
        prov.update_noise(float(final_noise))
    Xt = np.ascontiguousarray(x_test, dtype=np.float32)
    if Xt.ndim == 1:
        Xt = Xt[:, None]
    t2 = time.perf_counter()
    mean, var = cache.predict(Xt, return_var=variance_method == PREDICT_LOVE)
    mean_s = time.perf_counter() - t2
    exact_iters, var_s = 0, 0.0  # LOVE: the variance comes out of the mean's cross-product pass
    if variance_method == PREDICT_EXACT:
        t3 = time.perf_counter()
        var, exact_iters = prediction.exact_variance(prov, Xt, max_cg_iter, cg_tol, precond_rank,
                                                     exact_block_cols, comm=comm)
        var_s = time.perf_counter() - t3
    m = Xt.shape[0]
    var = np.zeros(m, np.float32) if var is None else np.asarray(var, dtype=np.float32)
    return {
        "mean": np.asarray(mean, dtype=np.float32),
        "variance": var,
        "std": np.sqrt(np.maximum(var, 0)).astype(np.float32),
        "mean_time_s": mean_s,
        "variance_time_s": var_s,
        "exact_cg_total_iterations": int(exact_iters),
        "provider_state_update_skipped": bool(provider_state_current),
    }


def prepare_prediction_cache(info, y, params, final_noise: float, final_mean: float,
                             variance_method: int, max_cg_iter: int = 100, cg_tol: float = 1e-2,
                             precond_rank: int = 10, lanczos_rank: int = 0,
                             provider_state_current: bool = False, cached_alpha=None,
                             cached_love_root=None, *, comm=None) -> dict:
    """Device-resident alpha and LOVE root for repeated predictions, with the
    reference binding's positional arguments and result keys
    (prepare_prediction_cache, jit_engine_bindings.mojo:636-768). The returned
    `cache_handle` goes to predict_with_cache / destroy_prediction_cache."""
    import time

    t = time.perf_counter()
    cache, _, f = _build_cache(info, y, params, final_noise, final_mean, variance_method,
                               max_cg_iter, cg_tol, lanczos_rank, provider_state_current,
                               cached_alpha, cached_love_root, comm)
    handle = int(cache.handle)
    _CACHES[handle] = cache
    return {"cache_handle": handle, "n_train": int(_provider_of(info).n), "rank": f["rank"],
            "has_love_root": f["rank"] > 0, "alpha_time_s": f["alpha_time_s"],
            "love_root_time_s": f["love_root_time_s"], "prepare_time_s": time.perf_counter() - t,
            "alpha_cache_used": f["alpha_cache_used"],
            "love_root_cache_used": f["love_root_cache_used"]}


def predict_with_cache(info, cache_handle: int, x_test, params, final_noise: float,
                       final_mean: float, variance_method: int, max_cg_iter: int = 100,
                       cg_tol: float = 1e-2, precond_rank: int = 10, lanczos_rank: int = 0,
                       provider_state_current: bool = False, exact_block_cols: int = 0,
                       test_info=None, *, comm=None) -> dict:
    """Prediction from a prepared cache (predict_with_cache,
    jit_engine_bindings.mojo:782-942): mean from the cached alpha, LOVE variance
    from the cached root, CG-exact variance on demand."""
    import time

    cache = _CACHES.get(int(cache_handle)) if cache_handle else None
    if cache is None:
        raise ValueError("predict_with_cache() received null or unknown cache handle")
    t = time.perf_counter()
    out = _predict_from_cache(info, cache, x_test, params, final_noise, variance_method,
                              max_cg_iter, cg_tol, precond_rank, provider_state_current,
                              exact_block_cols, comm)
    out.update({"alpha_time_s": 0.0, "love_root_time_s": 0.0,
                "total_time_s": time.perf_counter() - t, "alpha_cache_used": True,
                "love_root_cache_used": variance_method == PREDICT_LOVE and cache.rank > 0,
                "prediction_cache_used": True})
    return out


def destroy_prediction_cache(cache_handle: int) -> None:
    """Release a cache from prepare_prediction_cache (jit_engine_bindings.mojo:770-780)."""
    cache = _CACHES.pop(int(cache_handle), None)
    if cache is not None:
        cache.destroy()


def predict(info, y, x_test, params, final_noise: float, final_mean: float,
            variance_method: int, max_cg_iter: int = 100, cg_tol: float = 1e-2,
            precond_rank: int = 10, lanczos_rank: int = 0, provider_state_current: bool = False,
            exact_block_cols: int = 0, cached_alpha=None, cached_love_root=None, test_info=None,
            *, comm=None) -> dict:
    """Engine-level prediction with the reference binding's positional arguments
    and result keys (predict, jit_engine_bindings.mojo:944-1234).

    Unless `provider_state_current`, the provider takes `params` and
    `final_noise` first. alpha = (K + noise I)^{-1} (y - final_mean) by CG
    (`max_cg_iter`, `cg_tol`), or `cached_alpha`. variance_method 0: mean only;
    1: LOVE with a root of `lanczos_rank` vectors (<= 0: 100, 200 for ARD
    kernels), or `cached_love_root` [rank * n]; 2: CG-exact variance (blocks of
    `exact_block_cols`, preconditioner rank `precond_rank`). Variances include
    the noise. The result carries `cached_alpha` / `cached_lanczos_root` when
    they were computed here, for the caller to pass back. `test_info` is
    accepted for signature compatibility: test-point diagonals come from the
    training provider's kernel.
    """
    import time

    t_start = time.perf_counter()
    cache, alpha, f = _build_cache(info, y, params, final_noise, final_mean, variance_method,
                                   max_cg_iter, cg_tol, lanczos_rank, provider_state_current,
                                   cached_alpha, cached_love_root, comm)
    try:
        out = _predict_from_cache(info, cache, x_test, params, final_noise, variance_method,
                                  max_cg_iter, cg_tol, precond_rank, True, exact_block_cols, comm)
        root_out = cache.root() if (f["rank"] > 0 and not f["love_root_cache_used"]) else None
    finally:
        cache.destroy()
    out.update({"alpha_time_s": f["alpha_time_s"], "love_root_time_s": f["love_root_time_s"],
                "total_time_s": time.perf_counter() - t_start,
                "provider_state_update_skipped": bool(provider_state_current),
                "alpha_cache_used": f["alpha_cache_used"],
                "love_root_cache_used": f["love_root_cache_used"]})
    if not f["alpha_cache_used"]:
        out["cached_alpha"] = alpha
    if root_out is not None:
        out["cached_lanczos_root"] = root_out.ravel()
    return out
