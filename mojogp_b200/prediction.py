"""Prediction over the C ABI: alpha solve, LOVE prediction cache, mean/variance.

Mirrors the reference engine's predict / prepare_prediction_cache /
predict_with_cache / destroy_prediction_cache bindings
(mojogp/kernels/jit/jit_engine_bindings.mojo:636-1234).
"""
from __future__ import annotations

import ctypes as C
from typing import Optional

import numpy as np

from . import _lib
from .provider import Provider


def _p(a):
    return C.c_void_p(a.ctypes.data)


def compute_alpha(provider: Provider, y_centered: np.ndarray, max_cg_iter: int = 300,
                  cg_tol: float = 1e-3, comm=None):
    """(K + noise I)^{-1} (y - mean) by CG (relative-residual stop); returns (alpha, iters)."""
    y = np.ascontiguousarray(y_centered, dtype=np.float32).ravel()
    alpha = np.zeros(provider.n, np.float32)
    it = C.c_int32()
    _lib.call("gpb_compute_alpha", provider.h, C.c_void_p(comm.handle) if comm else None, _p(y),
              provider.n, int(max_cg_iter), float(cg_tol), _p(alpha), C.byref(it))
    return alpha, int(it.value)


def exact_variance(provider: Provider, X_test: np.ndarray, max_cg_iter: int = 300,
                   cg_tol: float = 1e-3, precond_rank: int = 0, block_cols: int = 0, comm=None):
    """CG-exact predictive variance (noise included) for every test point; returns
    (variance [m], total CG iterations over the blocks)."""
    Xt = np.ascontiguousarray(X_test, dtype=np.float32)
    if Xt.ndim == 1:
        Xt = Xt[:, None]
    var = np.zeros(Xt.shape[0], np.float32)
    it = C.c_int32()
    _lib.call("gpb_predict_exact_variance", provider.h, C.c_void_p(comm.handle) if comm else None,
              _p(Xt), Xt.shape[0], int(block_cols), int(max_cg_iter), float(cg_tol),
              int(precond_rank), _p(var), C.byref(it))
    return var, it.value


class PredictionCache:
    """Device-resident alpha and LOVE root S ([rank][n]) for repeated predictions."""

    def __init__(self, provider: Provider, alpha: np.ndarray, mean: float, love_rank: int,
                 root: Optional[np.ndarray] = None, comm=None):
        self.provider = provider
        self.rank = int(love_rank)
        a = np.ascontiguousarray(alpha, dtype=np.float32).ravel()
        r = None
        if root is not None:
            r = np.ascontiguousarray(root, dtype=np.float32).reshape(self.rank, provider.n)
        h = C.c_void_p()
        _lib.call("gpb_prediction_cache_create", provider.h,
                  C.c_void_p(comm.handle) if comm else None, _p(a), float(mean), self.rank,
                  _p(r) if r is not None else None, C.byref(h))
        self.handle = h.value
        self._keep = (a, r)

    def root(self) -> np.ndarray:
        out = np.zeros((self.rank, self.provider.n), np.float32)
        _lib.call("gpb_prediction_cache_root", C.c_void_p(self.handle), _p(out))
        return out

    def predict(self, X_test: np.ndarray, return_var: bool = True):
        Xt = np.ascontiguousarray(X_test, dtype=np.float32)
        if Xt.ndim == 1:
            Xt = Xt[:, None]
        if Xt.shape[1] != self.provider.d:
            raise ValueError(f"X_test has {Xt.shape[1]} columns, model has {self.provider.d}")
        mean = np.zeros(Xt.shape[0], np.float32)
        var = np.zeros(Xt.shape[0], np.float32) if (return_var and self.rank > 0) else None
        _lib.call("gpb_predict_with_cache", C.c_void_p(self.handle), _p(Xt), Xt.shape[0], _p(mean),
                  _p(var) if var is not None else None)
        return mean, var

    def predict_sharded(self, X_test: np.ndarray, comm, return_var: bool = True):
        """Each rank predicts its slice of the test rows (rows [m r / W, m (r+1) / W))
        with the replicated alpha / LOVE root; one all-reduce assembles the full
        outputs on every rank (X* sharding: no collective on the data path)."""
        Xt = np.ascontiguousarray(X_test, dtype=np.float32)
        if Xt.ndim == 1:
            Xt = Xt[:, None]
        m = Xt.shape[0]
        from .distributed import shard_bounds
        a, b = shard_bounds(m, comm.world, comm.rank)
        mean_l, var_l = self.predict(Xt[a:b], return_var=return_var) if b > a else \
            (np.zeros(0, np.float32), np.zeros(0, np.float32) if return_var else None)
        want_var = return_var and self.rank > 0
        buf = np.zeros(2 * m if want_var else m)
        buf[a:b] = mean_l
        if want_var:
            buf[m + a:m + b] = var_l
        buf = comm.allreduce_sum(buf)
        mean = buf[:m].astype(np.float32)
        var = buf[m:].astype(np.float32) if want_var else None
        return mean, var

    def destroy(self) -> None:
        if getattr(self, "handle", None):
            _lib.lib().gpb_prediction_cache_destroy(C.c_void_p(self.handle))
            self.handle = None

    def __del__(self):
        try:
            self.destroy()
        except Exception:
            pass
