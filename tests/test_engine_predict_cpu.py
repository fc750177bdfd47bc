"""engine.predict's orchestration (the reference binding's argument handling
and result keys, jit_engine_bindings.mojo:944-1234) with stand-ins for the
device calls (CPU): which provider updates, solves and caches run for each
variance method and cache argument, and the keys that come back."""
import inspect

import numpy as np
import pytest

from mojogp_b200 import engine, prediction


class _Prov:
    n = 6

    def __init__(self):
        self.calls = []

    def update_params(self, p):
        self.calls.append(("params", np.asarray(p).tolist()))

    def update_noise(self, s):
        self.calls.append(("noise", s))


class _Cache:
    made = []

    def __init__(self, provider, alpha, mean, love_rank, root=None, comm=None):
        _Cache.made.append(dict(alpha=np.asarray(alpha), mean=mean, rank=love_rank, root=root))
        self.rank, self.n = love_rank, provider.n
        self.destroyed = False
        self.handle = id(self)

    def predict(self, Xt, return_var=True):
        m = Xt.shape[0]
        return np.full(m, 1.5, np.float32), (np.full(m, 0.25, np.float32)
                                             if (return_var and self.rank > 0) else None)

    def root(self):
        return np.arange(self.rank * self.n, dtype=np.float32).reshape(self.rank, self.n)

    def destroy(self):
        self.destroyed = True


@pytest.fixture
def stubs(monkeypatch):
    log = {}

    def compute_alpha(provider, y_centered, max_cg_iter=300, cg_tol=1e-3, comm=None):
        log["alpha"] = (np.asarray(y_centered).tolist(), max_cg_iter, cg_tol)
        return np.full(provider.n, 2.0, np.float32), 7

    def exact_variance(provider, X_test, max_cg_iter=300, cg_tol=1e-3, precond_rank=0,
                       block_cols=0, comm=None):
        log["exact"] = (max_cg_iter, cg_tol, precond_rank, block_cols)
        return np.full(X_test.shape[0], 0.5, np.float32), 11

    # The stand-ins take the real functions' parameters, in order.
    names = lambda f: list(inspect.signature(f).parameters)
    assert names(compute_alpha) == names(prediction.compute_alpha)
    assert names(exact_variance) == names(prediction.exact_variance)
    assert names(_Cache.__init__) == names(prediction.PredictionCache.__init__)
    monkeypatch.setattr(prediction, "compute_alpha", compute_alpha)
    monkeypatch.setattr(prediction, "exact_variance", exact_variance)
    monkeypatch.setattr(prediction, "PredictionCache", _Cache)
    _Cache.made = []
    return log


def _info(ard=False):
    return {"provider": _Prov(), "n": 6, "is_ard": ard}


def test_love_route_computes_alpha_and_root(stubs):
    info = _info()
    y = np.arange(6, dtype=np.float32)
    out = engine.predict(info, y, np.zeros((3, 2)), np.array([0.5, 1.0]), 0.1, 2.0, 1, 50, 1e-3)
    assert info["provider"].calls == [("params", [0.5, 1.0]), ("noise", 0.1)]
    assert stubs["alpha"] == ((y - 2.0).tolist(), 50, 1e-3)
    assert _Cache.made[0]["rank"] == 6  # default 100 capped at n
    assert out["mean"].tolist() == [1.5] * 3 and out["variance"].tolist() == [0.25] * 3
    np.testing.assert_allclose(out["std"], 0.5)
    assert out["cached_alpha"].tolist() == [2.0] * 6
    assert out["cached_lanczos_root"].shape == (36,)
    assert not out["alpha_cache_used"] and not out["love_root_cache_used"]
    for k in ("alpha_time_s", "mean_time_s", "variance_time_s", "love_root_time_s",
              "total_time_s", "provider_state_update_skipped"):
        assert k in out


def test_caches_and_state_flags_are_honoured(stubs):
    info = _info()
    root = np.ones(6 * 4, np.float32)
    out = engine.predict(info, np.zeros(6), np.zeros((2, 2)), [1.0, 1.0], 0.1, 0.0, 1, 100, 1e-2,
                         10, 4, True, 0, np.full(6, 3.0), root)
    assert info["provider"].calls == []  # provider_state_current
    assert "alpha" not in stubs and _Cache.made[0]["alpha"].tolist() == [3.0] * 6
    assert _Cache.made[0]["rank"] == 4 and _Cache.made[0]["root"].shape == (4, 6)
    assert out["alpha_cache_used"] and out["love_root_cache_used"]
    assert "cached_alpha" not in out and "cached_lanczos_root" not in out
    assert out["provider_state_update_skipped"]


def test_exact_and_mean_only_routes(stubs):
    out = engine.predict(_info(), np.zeros(6), np.zeros((4, 2)), [1.0, 1.0], 0.1, 0.0, 2, 120,
                         5e-3, 15, 0, False, 64)
    assert stubs["exact"] == (120, 5e-3, 15, 64)
    assert _Cache.made[0]["rank"] == 0
    assert out["variance"].tolist() == [0.5] * 4 and out["exact_cg_total_iterations"] == 11
    assert "cached_lanczos_root" not in out
    out = engine.predict(_info(), np.zeros(6), np.zeros((4, 2)), [1.0, 1.0], 0.1, 0.0, 0)
    assert out["variance"].tolist() == [0.0] * 4 and out["std"].tolist() == [0.0] * 4
    with pytest.raises(ValueError):
        engine.predict(_info(), np.zeros(6), np.zeros((1, 2)), [1.0, 1.0], 0.1, 0.0, 3)


def test_love_rank_default_for_ard(stubs):
    info = _info(ard=True)
    info["provider"].n = 1000
    engine.predict(info, np.zeros(1000), np.zeros((1, 2)), [1.0] * 3, 0.1, 0.0, 1)
    assert _Cache.made[0]["rank"] == 200


def test_train_binding_maps_the_reference_positional_arguments(monkeypatch):
    """engine.train_binding takes the reference engine's positional layout
    (jit_engine_bindings.mojo:123-247) and forwards it to engine.train."""
    seen = {}

    def fake_train(provider, y, **kw):
        seen.update(kw)
        return {"final_nll": 0.5, "noise": 0.1, "mean": 0.0, "iterations": 3, "converged": False,
                "params": np.ones(2, np.float32), "iter_times_ms": np.ones(3),
                "nll_history": np.ones(3), "cg_iterations_history": np.ones(3, np.int32),
                "cached_alpha": None, "precond_build_count": 2, "precond_build_time_ms": 4.0,
                "precond_rank": 12}

    monkeypatch.setattr(engine, "train", fake_train)
    info = {"provider": _Prov(), "materialization_mode": 1, "is_ard": True}
    args = (info, np.zeros(6), np.array([0.7, 1.3]), 0.2, 40, 0.05, 15, 120, 1e-3, 12, False,
            False, True, 25, 0.4, 0, 0.3, True, 7, 1e-5, False)
    out = engine.train_binding(*args)
    assert info["provider"].calls == [("params", [pytest.approx(0.7), pytest.approx(1.3)]),
                                      ("noise", 0.2)]
    assert seen == {"max_iterations": 40, "learning_rate": 0.05, "num_probes": 15,
                    "max_cg_iter": 120, "cg_tol": 1e-3, "precond_rank": 12,
                    "max_tridiag_iter": 25, "precond_rebuild_threshold": 0.4,
                    "use_cosine_lr": False, "use_preconditioner": True, "learn_noise": False,
                    "init_mean": 0.3, "enable_early_stopping": True, "early_stop_patience": 7,
                    "early_stop_tol": 1e-5, "verbose": False, "trainable_mask": None,
                    "comm": None}
    assert out["training_route"] == "materialized" and out["precond_rebuild_count"] == 1
    assert out["actual_precond_rank"] == 12 and out["precond_build_total_ms"] == 4.0
    for k in ("final_nll", "noise", "mean", "iterations", "converged", "params", "iter_times_ms",
              "nll_history", "cg_iterations_history", "cached_alpha", "use_preconditioner",
              "precond_method", "learn_noise", "is_ard"):
        assert k in out
    with pytest.raises(NotImplementedError):
        engine.train_binding(info, np.zeros(6), [1.0, 1.0], 0.1, 5, 0.01, 10, 100, 1e-2, 10,
                             False, False, True, 30, 0.5, 2, 0.0)


def test_prepared_cache_round_trip(stubs):
    """prepare_prediction_cache -> predict_with_cache (several times) ->
    destroy_prediction_cache, with the reference bindings' keys."""
    info = _info()
    prep = engine.prepare_prediction_cache(info, np.ones(6), [1.0, 1.0], 0.1, 1.0, 1, 80, 1e-3,
                                           10, 3, False)
    assert prep["rank"] == 3 and prep["has_love_root"] and prep["n_train"] == 6
    assert not prep["alpha_cache_used"] and stubs["alpha"][1:] == (80, 1e-3)
    h = prep["cache_handle"]
    for _ in range(2):
        out = engine.predict_with_cache(info, h, np.zeros((5, 2)), [1.0, 1.0], 0.1, 1.0, 1,
                                        provider_state_current=True)
        assert out["variance"].tolist() == [0.25] * 5 and out["prediction_cache_used"]
        assert out["love_root_cache_used"] and out["alpha_cache_used"]
    out = engine.predict_with_cache(info, h, np.zeros((2, 2)), [1.0, 1.0], 0.1, 1.0, 2, 90, 1e-4,
                                    5, 0, True, 32)
    assert stubs["exact"] == (90, 1e-4, 5, 32) and out["variance"].tolist() == [0.5, 0.5]
    cache = engine._CACHES[h]
    engine.destroy_prediction_cache(h)
    assert cache.destroyed and h not in engine._CACHES
    with pytest.raises(ValueError, match="cache handle"):
        engine.predict_with_cache(info, h, np.zeros((1, 2)), [1.0, 1.0], 0.1, 1.0, 1)
    engine.destroy_prediction_cache(h)  # a second destroy is harmless
