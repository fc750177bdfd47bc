"""Input / target standardisation (mojogp/utils.py:11-173: StandardScaler).

Features are centred and divided by their standard deviation (constant
features keep scale 1); targets likewise. Predictions map back with
mean * y_std + y_mean, std * y_std and variance * y_std^2. Statistics are
float64; transformed arrays are float32.
"""
from __future__ import annotations

from typing import Optional

import numpy as np


class StandardScaler:
    def __init__(self):
        self.X_mean_: Optional[np.ndarray] = None
        self.X_std_: Optional[np.ndarray] = None
        self.y_mean_: Optional[float] = None
        self.y_std_: Optional[float] = None
        self._is_fitted = False

    def fit(self, X: np.ndarray, y: Optional[np.ndarray] = None) -> "StandardScaler":
        X = np.asarray(X, dtype=np.float64)
        self.X_mean_ = X.mean(axis=0)
        sd = X.std(axis=0)
        self.X_std_ = np.where(sd < 1e-12, 1.0, sd)
        if y is not None:
            y = np.asarray(y, dtype=np.float64)
            self.y_mean_ = float(y.mean())
            s = float(y.std())
            self.y_std_ = 1.0 if s < 1e-12 else s
        self._is_fitted = True
        return self

    def _need(self, y: bool = False) -> None:
        if not self._is_fitted:
            raise RuntimeError("Call fit() or fit_transform() first")
        if y and self.y_mean_ is None:
            raise RuntimeError("Scaler was not fitted with y data")

    def transform_X(self, X: np.ndarray) -> np.ndarray:
        self._need()
        return ((np.asarray(X, dtype=np.float64) - self.X_mean_) / self.X_std_).astype(np.float32)

    def transform_y(self, y: np.ndarray) -> np.ndarray:
        self._need(y=True)
        return ((np.asarray(y, dtype=np.float64) - self.y_mean_) / self.y_std_).astype(np.float32)

    def fit_transform(self, X: np.ndarray, y: Optional[np.ndarray] = None) -> tuple:
        """(X_scaled,) or, with y, (X_scaled, y_scaled)."""
        self.fit(X, y)
        if y is None:
            return (self.transform_X(X),)
        return self.transform_X(X), self.transform_y(y)

    def inverse_transform_y(self, mean: np.ndarray, std: Optional[np.ndarray] = None,
                            variance: Optional[np.ndarray] = None) -> tuple:
        """(mean,), (mean, std) or (mean, variance) in the original scale; std wins
        when both are given."""
        self._need(y=True)
        m = (np.asarray(mean, dtype=np.float64) * self.y_std_ + self.y_mean_).astype(np.float32)
        if std is not None:
            return m, (np.asarray(std, dtype=np.float64) * self.y_std_).astype(np.float32)
        if variance is not None:
            return m, (np.asarray(variance, dtype=np.float64) * self.y_std_ ** 2).astype(np.float32)
        return (m,)

    def inverse_transform_X(self, X: np.ndarray) -> np.ndarray:
        self._need()
        return (np.asarray(X, dtype=np.float64) * self.X_std_ + self.X_mean_).astype(np.float32)
