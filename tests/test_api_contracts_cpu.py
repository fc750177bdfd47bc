"""Public-API argument contracts that hold before any device work (CPU): the
reference's validation order and messages for the fits
(mojogp/gp.py:995-1004, 1266-1284; multi_output_gp.py:1542-1615, 4659-4675)
and the untrained-predict error. Restated from the reference's contract tests
(tests/unit/test_gp_wrapper_api_contracts.py:44-100)."""
import numpy as np
import pytest

from mojogp_b200.gp import SingleOutputGP
from mojogp_b200.kernel import RBF
from mojogp_b200.multi_output_gp import MultiOutputGP, MultiOutputLMCGP


@pytest.fixture
def data():
    rng = np.random.default_rng(0)
    X = rng.uniform(-1, 1, size=(40, 2)).astype(np.float32)
    Y = rng.standard_normal((40, 3)).astype(np.float32)
    return X, Y


def _models():
    return [("icm", lambda: MultiOutputGP(kernel="rbf")),
            ("lmc", lambda: MultiOutputLMCGP(kernels=["rbf"]))]


@pytest.mark.parametrize("name,make", _models())
def test_multi_output_rejects_non_finite_data(data, name, make):
    X, Y = data
    Xb = X.copy()
    Xb[0, 0] = np.nan
    with pytest.raises(ValueError, match="X contains NaN or Inf"):
        make().fit(Xb, Y, max_iterations=5)
    Yb = Y.copy()
    Yb[1, 2] = np.inf
    with pytest.raises(ValueError, match="Y contains NaN or Inf"):
        make().fit(X, Yb, max_iterations=5)


@pytest.mark.parametrize("name,make", _models())
@pytest.mark.parametrize("kw,msg", [({"initial_noise": -0.1}, "initial_noise must be > 0"),
                                    ({"learning_rate": 0.0}, "learning_rate must be > 0"),
                                    ({"learning_rate": -0.01}, "learning_rate must be > 0"),
                                    ({"max_iterations": 0}, "max_iterations must be > 0")])
def test_multi_output_rejects_bad_controls(data, name, make, kw, msg):
    X, Y = data
    with pytest.raises(ValueError, match=msg):
        make().fit(X, Y, **kw)


@pytest.mark.parametrize("name,make", _models())
def test_multi_output_shape_checks(data, name, make):
    X, Y = data
    with pytest.raises(ValueError, match="Y must be 2D"):
        make().fit(X, Y[:, 0])
    with pytest.raises(ValueError, match="samples"):
        make().fit(X, Y[:30])
    with pytest.raises(ValueError, match="X must be 2D"):
        make().fit(X[:, 0], Y)


@pytest.mark.parametrize("name,make", _models())
def test_multi_output_predict_before_fit(data, name, make):
    with pytest.raises(RuntimeError, match="trained"):
        make().predict(data[0])


def test_single_output_contracts(data):
    X, Y = data
    y = Y[:, 0]
    gp = SingleOutputGP(RBF())
    with pytest.raises(ValueError, match="X contains NaN or Inf"):
        Xb = X.copy()
        Xb[3, 1] = np.inf
        gp.fit(Xb, y)
    with pytest.raises(ValueError, match="y contains NaN or Inf"):
        yb = y.copy()
        yb[0] = np.nan
        gp.fit(X, yb)
    with pytest.raises(ValueError, match="samples"):
        gp.fit(X, y[:10])
    with pytest.raises(ValueError, match="2D"):
        gp.fit(X[:, 0], y)
    with pytest.raises(ValueError, match="y must be 1D"):
        gp.fit(X, Y)
    with pytest.raises(ValueError, match="max_iterations must be > 0"):
        gp.fit(X, y, max_iterations=0)
    with pytest.raises(ValueError, match="learning_rate must be > 0"):
        gp.fit(X, y, learning_rate=0.0)
    with pytest.raises(ValueError, match="initial_noise must be > 0"):
        gp.fit(X, y, initial_noise=-0.1)
    with pytest.raises(ValueError, match="Unknown preset"):
        gp.fit(X, y, preset="turbo")
    with pytest.raises(ValueError, match="lr_schedule"):
        gp.fit(X, y, lr_schedule="linear")
    with pytest.raises(ValueError, match="method"):
        gp.fit(X, y, method="bogus")
    with pytest.raises(RuntimeError, match="trained"):
        gp.predict(X)
    with pytest.raises(RuntimeError, match="trained"):
        gp.get_learned_params()


def _route(method, n, dim, kt, ard=False, lr=0.01, default=True, **kw):
    from mojogp_b200.gp import _resolve_fit_route
    args = dict(preconditioner=None, preconditioner_rank=None, use_preconditioner=None,
                precond_rebuild_threshold=None)
    args.update(kw)
    return _resolve_fit_route(method, n, dim, kt, ard, lr, default,
                              np.ones(3, np.float32), **args)


def test_fit_route_defaults_follow_the_reference():
    """SingleOutputGP.fit's route resolution and route defaults
    (mojogp/gp.py:1350-1468)."""
    from mojogp_b200.kernel import KernelType as K
    # auto: the dense route up to 2000 rows
    assert _route("auto", 2000, 1, K.RBF)["method"] == "materialized"
    assert _route("auto", 2001, 1, K.RBF)["method"] == "matrix_free"
    assert _route("mat", 10, 1, K.RBF)["method"] == "materialized"
    # dense 1-D RBF starts at lengthscale 0.5; the preset's preconditioner rank
    r = _route("materialized", 500, 1, K.RBF)
    assert r["params"][0] == np.float32(0.5) and r["precond_rank"] is None
    assert _route("materialized", 500, 1, K.RBF, lr=0.1)["params"][0] == 1.0
    assert _route("materialized", 500, 1, K.RBF, default=False)["params"][0] == 1.0
    assert _route("materialized", 500, 2, K.RBF)["params"][0] == 1.0
    # dense Matérn-3/2 greedy; dense Linear unpreconditioned; dense ARD threshold 0.1
    assert _route("materialized", 500, 2, K.MATERN32)["preconditioner"] == "greedy"
    assert _route("materialized", 500, 2, K.LINEAR)["precond_rank"] == 0
    assert _route("materialized", 500, 2, K.LINEAR, preconditioner_rank=7)["precond_rank"] == 7
    assert _route("materialized", 500, 3, K.MATERN52, ard=True)["precond_rebuild_threshold"] == 0.1
    assert _route("materialized", 500, 3, None, ard=True)["precond_rebuild_threshold"] is None
    # matrix-free: low-d isotropic RBF gets the milder start and rank 256 ...
    r = _route("matrix_free", 20000, 4, K.RBF)
    assert r["params"][0] == np.float32(0.6)
    assert (r["preconditioner"], r["precond_rank"]) == ("greedy", 256)
    r = _route("matrix_free", 6000, 4, K.RBF)
    assert r["params"][0] == 1.0 and r["precond_rank"] == 256
    # ... everything else runs unpreconditioned unless asked
    assert _route("matrix_free", 20000, 9, K.RBF)["precond_rank"] == 0
    assert _route("matrix_free", 20000, 4, K.RBF, ard=True)["precond_rank"] == 0
    assert _route("matrix_free", 20000, 4, K.MATERN52)["precond_rank"] == 0
    assert _route("matrix_free", 20000, 4, K.MATERN52, preconditioner="greedy")["precond_rank"] is None
    assert _route("matrix_free", 20000, 4, K.RBF, use_preconditioner=False)["precond_rank"] is None


def test_standard_scaler_round_trip():
    from mojogp_b200 import StandardScaler
    rng = np.random.default_rng(3)
    X = rng.normal(5.0, 3.0, size=(200, 3))
    X[:, 2] = 7.0  # constant feature keeps scale 1
    y = rng.normal(-2.0, 0.5, size=200)
    sc = StandardScaler()
    Xs, ys = sc.fit_transform(X, y)
    assert Xs.dtype == np.float32 and ys.dtype == np.float32
    np.testing.assert_allclose(Xs[:, :2].mean(0), 0, atol=1e-5)
    np.testing.assert_allclose(Xs[:, :2].std(0), 1, atol=1e-5)
    assert np.all(Xs[:, 2] == 0) and sc.X_std_[2] == 1.0
    np.testing.assert_allclose(sc.inverse_transform_X(Xs), X, rtol=1e-5, atol=1e-5)
    m, s = sc.inverse_transform_y(ys, std=np.ones(200))
    np.testing.assert_allclose(m, y, rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(s, y.std(), rtol=1e-6)
    _, v = sc.inverse_transform_y(ys, variance=np.ones(200))
    np.testing.assert_allclose(v, y.std() ** 2, rtol=1e-6)
    assert len(sc.inverse_transform_y(ys)) == 1
    only_x = StandardScaler()
    assert len(only_x.fit_transform(X)) == 1
    with pytest.raises(RuntimeError, match="not fitted with y"):
        only_x.transform_y(y)
    with pytest.raises(RuntimeError, match="fit"):
        StandardScaler().transform_X(X)


def test_fit_gp_validates_before_device_work():
    from mojogp_b200 import RBF, fit_gp
    with pytest.raises(ValueError, match="max_iterations must be > 0"):
        fit_gp(np.zeros((4, 2), np.float32), np.zeros(4, np.float32), RBF(), max_iterations=0)


def test_multi_output_prediction_return_convention():
    """No flags: a MultiOutputPredictionResult (multi_output_gp.py:545-550);
    return_std / return_var: tuples; mean-only variance is zeros in a tuple and
    None in the result object."""
    from mojogp_b200.multi_output_gp import MultiOutputPredictionResult, _prediction_output
    mean = np.ones((3, 2), np.float32)
    var = np.full((3, 2), 4.0, np.float32)
    r = _prediction_output(mean, var, False, False)
    assert isinstance(r, MultiOutputPredictionResult)
    assert np.all(r.std == 2.0) and r.variance is var and r.mean is mean
    assert _prediction_output(mean, var, True, False)[1] is var
    assert np.all(_prediction_output(mean, var, False, True)[1] == 2.0)
    assert np.all(_prediction_output(mean, var, True, True)[1] == 2.0)
    r = _prediction_output(mean, None, False, False)
    assert r.variance is None and r.std is None
    assert np.all(_prediction_output(mean, None, True, False)[1] == 0)


def test_fitted_models_answer_for_the_reference_result_fields():
    """fit() returns the model; its properties give the reference result
    objects' fields (LMCTrainingResult, MultiOutputTrainingResult) from the
    attributes the fit loop sets. Populated here by hand (no device)."""
    from mojogp_b200.kernel import Matern32, make_ard_kernel
    lmc = object.__new__(MultiOutputLMCGP)
    T, n = 2, 5
    lmc.T, lmc.ard = T, True
    lmc.kernels_resolved = [make_ard_kernel(RBF(ard=True), 2), Matern32().resolve_ard(2)]
    lmc.params_ = [np.array([0.5, 0.7, 1.5]), np.array([0.9, 2.0])]
    lmc.A = np.stack([np.eye(T), 2 * np.eye(T)])
    lmc.noise = np.array([0.1, 0.2])
    lmc.mean_ = np.array([1.0, -1.0])
    lmc.nll_history = np.array([3.0, 2.0, 1.5])
    lmc._alpha = np.arange(T * n, dtype=np.float32)
    assert lmc.num_tasks == 2 and lmc.iterations == 3 and lmc.converged is False
    np.testing.assert_array_equal(lmc.B, 3 * np.eye(T))
    np.testing.assert_allclose(lmc.Lambda, [3.0, 3.0])
    assert lmc.alpha.shape == (n, T) and lmc.alpha[1, 1] == n + 1
    np.testing.assert_allclose(lmc.lengthscales, [0.5, 0.7, 0.9])
    np.testing.assert_allclose(lmc.outputscales, [1.5, 2.0])
    np.testing.assert_array_equal(lmc.noise_per_task, [0.1, 0.2])
    assert lmc.use_ard and len(lmc.params_per_latent) == 2
    icm = object.__new__(MultiOutputGP)
    icm.T = 3
    icm.noise_per_task = np.array([0.1, 0.2, 0.3])
    icm.params_ = np.array([0.8, 1.0], np.float32)
    icm.task_covariance = np.diag([1.0, 2.0, 3.0])
    icm._Q, icm._Lambda = np.eye(3), np.array([1.0, 2.0, 3.0])
    icm.W_ = np.ones((3, 1))
    icm.mean_ = np.zeros(3)
    icm.nll_history = np.array([1.0, 0.5])
    assert icm.num_tasks == 3 and icm.iterations == 2 and icm.num_kernel_params == 2
    assert icm.noise == pytest.approx(0.2)
    np.testing.assert_array_equal(icm.B, icm.task_covariance)
    np.testing.assert_array_equal(icm.effective_scales, [1.0, 2.0, 3.0])
    assert icm.W.shape == (3, 1) and icm.params.shape == (2,)


def _trained_stub():
    from mojogp_b200.gp import TrainingResult
    gp = SingleOutputGP(RBF())
    gp.dim = 2
    gp._training_result = TrainingResult(params=np.ones(2, np.float32), noise=0.1, mean=0.0,
                                         nll=1.0, iterations=1, converged=False,
                                         nll_history=np.array([1.0]))
    return gp


def test_single_output_predict_argument_checks():
    """Checks that precede any device work (gp.py:2500-2525)."""
    gp = _trained_stub()
    X = np.zeros((3, 2), np.float32)
    with pytest.raises(ValueError, match="Only one of return_var or return_std"):
        gp.predict(X, return_var=True, return_std=True)
    with pytest.raises(ValueError, match="variance_method"):
        gp.predict(X, variance_method="fast")
    with pytest.raises(ValueError, match="target must be"):
        gp.predict(X, target="both")
    with pytest.raises(ValueError, match="exact_prediction_block_cols"):
        gp.predict(X, exact_prediction_block_cols=0)
    with pytest.raises(ValueError, match="features"):
        gp.predict(np.zeros((3, 5), np.float32))
    with pytest.raises(ValueError, match="X_test contains NaN"):
        gp.predict(np.full((3, 2), np.nan, np.float32))
    assert gp.is_trained and gp.nll_history.tolist() == [1.0]
    assert gp.param_names == ["rbf_lengthscale", "rbf_outputscale"] and gp.num_params == 2
    with pytest.raises(RuntimeError, match="scoring"):
        SingleOutputGP(RBF()).score(X, np.zeros(3))


def test_observation_noise_checks():
    from mojogp_b200.gp import _checked_observation_noise
    np.testing.assert_allclose(_checked_observation_noise([0.1, 0.2], 2), [0.1, 0.2], rtol=1e-7)
    with pytest.raises(ValueError, match="requires observation_noise"):
        _checked_observation_noise(None, 2)
    with pytest.raises(ValueError, match=r"shape \(2,\)"):
        _checked_observation_noise(np.ones(3), 2)
    with pytest.raises(ValueError, match="NaN or Inf"):
        _checked_observation_noise([np.inf, 0.1], 2)
    with pytest.raises(ValueError, match="noise_floor"):
        _checked_observation_noise([0.0, 0.1], 2)


def test_multi_output_observed_prediction_helpers():
    from mojogp_b200.multi_output_gp import (MultiOutputPredictionResult, _observed_noise_matrix,
                                             _observed_output)
    noise = _observed_noise_matrix(2, 3, np.full((2, 3), 0.5))
    lat = MultiOutputPredictionResult(mean=np.zeros((2, 3)), variance=np.full((2, 3), 1.5))
    r = _observed_output(lat, noise, False, False)
    np.testing.assert_allclose(r.variance, 2.0) and np.testing.assert_allclose(r.std, np.sqrt(2))
    assert _observed_output(lat, noise, True, False)[1].shape == (2, 3)
    with pytest.raises(ValueError, match="requires explicit observation_noise"):
        _observed_noise_matrix(2, 3, None)
    with pytest.raises(ValueError, match=r"shape \(2, 3\)"):
        _observed_noise_matrix(2, 3, np.ones(2))
    with pytest.raises(ValueError, match="> 0"):
        _observed_noise_matrix(2, 3, np.zeros((2, 3)))
    gp = MultiOutputLMCGP(kernels=["rbf"])
    with pytest.raises(RuntimeError, match="trained"):
        gp.predict_observed(np.zeros((2, 2)), np.ones((2, 3)))
    with pytest.raises(NotImplementedError):
        gp.predict_observed(np.zeros((2, 2)), noise_group_test=np.zeros(2))


def test_multi_output_trained_state_members():
    gp = MultiOutputLMCGP(kernels=["rbf"])
    assert gp.is_trained is False and gp.training_result is None
    assert gp.task_covariance is None
    with pytest.raises(RuntimeError, match="scoring"):
        gp.score(np.zeros((2, 2)), np.zeros((2, 2)))
    icm = MultiOutputGP(kernel="rbf")
    assert icm.is_trained is False and icm.training_result is None
