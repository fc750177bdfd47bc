"""Prediction (alpha CG, LOVE root, mean/variance) vs the float64 oracle.

Bar: predictive mean and std within 1e-4 (relative to the output scale);
variance is the LOVE estimate including the noise term."""
import numpy as np
import pytest

from mojogp_b200 import prediction
from mojogp_b200.kernel import RBF, Matern52, make_ard_kernel
from mojogp_b200.provider import Provider
from oracle import love as ol

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("kind", ["rbf_ard", "m52"])
def test_love_prediction_vs_oracle(gpb_lib, kind):
    rng = np.random.default_rng(3)
    n, d, nt, r = 600, 2, 150, 60
    X = rng.uniform(0, 1, size=(n, d)).astype(np.float32)
    y = (np.sin(5 * X[:, 0]) + 0.1 * rng.standard_normal(n)).astype(np.float32)
    Xs = rng.uniform(-0.1, 1.1, size=(nt, d)).astype(np.float32)
    if kind == "rbf_ard":
        k = make_ard_kernel(RBF(ard=True), d)
        p = np.array([0.4, 0.6, 1.1], np.float32)
    else:
        k = Matern52()
        p = np.array([0.5, 1.0], np.float32)
    noise, mean = 0.05, float(y.mean())
    prov = Provider(X, k, p, noise)
    # A tight alpha tolerance so the float32 and float64 solves agree to the
    # 1e-4 mean bar (at the default 1e-3 the solves themselves differ by ~1e-3).
    alpha, it = prediction.compute_alpha(prov, y - mean, 1000, 1e-5)
    cache = prediction.PredictionCache(prov, alpha, mean, r)
    mu, var = cache.predict(Xs)
    rmu, rvar, ralpha, _ = ol.predict(k.to_spec(d), p, X, y, noise, mean, Xs, r, max_cg=1000,
                                      tol=1e-5)
    assert np.abs(mu - rmu).max() < 1e-4 * max(np.abs(rmu).max(), 1.0)
    np.testing.assert_allclose(np.sqrt(var), np.sqrt(rvar), rtol=1e-4, atol=1e-5)
    # a supplied root reproduces the computed one exactly
    cache2 = prediction.PredictionCache(prov, alpha, mean, r, root=cache.root())
    mu2, var2 = cache2.predict(Xs)
    np.testing.assert_array_equal(mu2, mu)
    np.testing.assert_array_equal(var2, var)


def test_alpha_cg_vs_oracle(gpb_lib):
    rng = np.random.default_rng(4)
    n, d = 500, 3
    X = rng.uniform(0, 1, size=(n, d)).astype(np.float32)
    y = rng.standard_normal(n).astype(np.float32)
    k = make_ard_kernel(RBF(ard=True), d)
    p = np.array([0.5, 0.5, 0.5, 1.0], np.float32)
    prov = Provider(X, k, p, 0.2)
    alpha, it = prediction.compute_alpha(prov, y, 300, 1e-6)
    from oracle import kernels as ok
    A = ok.kernel_matrix(k.to_spec(d), p, X) + 0.2 * np.eye(n)
    ref = np.linalg.solve(A, y.astype(np.float64))
    assert np.linalg.norm(alpha - ref) / np.linalg.norm(ref) < 1e-4
    # The relative-residual stop rule holds on the device result.
    _, it3 = prediction.compute_alpha(prov, y, 300, 1e-3)
    assert 1 <= it3 < 300


def test_mean_only_cache(gpb_lib):
    rng = np.random.default_rng(5)
    n, d = 300, 2
    X = rng.uniform(size=(n, d)).astype(np.float32)
    prov = Provider(X, RBF(), np.array([0.5, 1.0], np.float32), 0.1)
    alpha = rng.standard_normal(n).astype(np.float32)
    cache = prediction.PredictionCache(prov, alpha, 0.5, 0)
    mu, var = cache.predict(X[:10])
    assert var is None
    from oracle import kernels as ok
    ref = ok.kernel_matrix(RBF().to_spec(d), np.array([0.5, 1.0]), X[:10], X) @ alpha + 0.5
    np.testing.assert_allclose(mu, ref, rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("rank,block", [(0, 0), (20, 37)])
def test_exact_variance_vs_dense(gpb_lib, rank, block):
    """CG-exact variance (predict_variance_exact_jit) against the dense formula
    k** - k*^T (K + noise I)^{-1} k* + noise; ragged blocks of 37 test points."""
    from oracle import kernels as ok
    rng = np.random.default_rng(8)
    n, d, nt = 700, 3, 100
    X = rng.uniform(0, 1, size=(n, d)).astype(np.float32)
    Xs = rng.uniform(-0.1, 1.1, size=(nt, d)).astype(np.float32)
    k = make_ard_kernel(RBF(ard=True), d)
    p = np.array([0.4, 0.6, 0.8, 1.2], np.float32)
    noise = 0.05
    prov = Provider(X, k, p, noise)
    var, iters = prediction.exact_variance(prov, Xs, max_cg_iter=1000, cg_tol=1e-6,
                                           precond_rank=rank, block_cols=block)
    spec = k.to_spec(d)
    K = ok.kernel_matrix(spec, p, X.astype(np.float64))
    Kx = ok.kernel_matrix(spec, p, Xs.astype(np.float64), X.astype(np.float64))
    kss = np.diag(ok.kernel_matrix(spec, p, Xs.astype(np.float64)))
    ref = np.maximum(kss - np.einsum("ij,ji->i", Kx, np.linalg.solve(K + noise * np.eye(n), Kx.T)),
                     1e-10) + noise
    assert iters > 0
    np.testing.assert_allclose(var, ref, rtol=1e-3, atol=1e-5)


def test_gp_predict_exact_route(gpb_lib):
    from mojogp_b200.gp import SingleOutputGP
    rng = np.random.default_rng(2)
    X = np.linspace(-3, 3, 400, dtype=np.float32)[:, None]
    y = (np.sin(2 * X[:, 0]) + 0.05 * rng.standard_normal(400)).astype(np.float32)
    gp = SingleOutputGP(RBF())
    gp.fit(X, y, max_iterations=10, method="matrix_free")
    Xs = np.linspace(-4, 4, 64, dtype=np.float32)[:, None]
    m_e, v_e = gp.predict(Xs, return_var=True, variance_method="exact", cg_tolerance=1e-5)
    # A root of rank 100: far past this 1-D kernel's numerical rank at this
    # noise, but short of n, where fp32 Lanczos continues on rounding noise once
    # the Krylov space is exhausted and the result turns on rounding details.
    m_l, v_l = gp.predict(Xs, return_var=True, variance_method="love",
                          max_root_decomposition_size=100, cg_tolerance=1e-5)
    # same alpha solve settings: the mean does not depend on the variance route
    np.testing.assert_allclose(m_e, m_l, rtol=0, atol=1e-6)
    np.testing.assert_allclose(v_e, v_l, rtol=2e-2, atol=1e-4)
    with pytest.raises(ValueError):
        gp.predict(Xs, variance_method="bogus")


def test_engine_predict_matches_model_predict(gpb_lib):
    """engine.predict (the reference binding's call shape and keys) gives the
    model API's LOVE prediction, and replays it bit for bit from the alpha and
    root it hands back."""
    from mojogp_b200 import engine, synthetic
    from mojogp_b200.gp import SingleOutputGP
    X, y, Xs = synthetic.config1()
    X, y = X[::4], y[::4]
    gp = SingleOutputGP(RBF())
    tr = gp.fit(X, y, max_iterations=5, method="matrix_free")
    m_ref, v_ref = gp.predict(Xs, return_var=True, max_root_decomposition_size=100,
                              max_cg_iterations=300, cg_tolerance=1e-3)
    info = {"provider": gp._provider, "n": X.shape[0], "is_ard": False}
    out = engine.predict(info, y, Xs, tr.params, tr.noise, tr.mean, engine.PREDICT_LOVE, 300,
                         1e-3, 10, 100)
    np.testing.assert_allclose(out["mean"], m_ref, rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(out["variance"], v_ref, rtol=1e-4, atol=1e-6)
    assert out["cached_lanczos_root"].shape == (100 * X.shape[0],)
    again = engine.predict(info, y, Xs, tr.params, tr.noise, tr.mean, engine.PREDICT_LOVE, 300,
                           1e-3, 10, 100, True, 0, out["cached_alpha"], out["cached_lanczos_root"])
    assert again["alpha_cache_used"] and again["love_root_cache_used"]
    np.testing.assert_array_equal(again["mean"], out["mean"])
    np.testing.assert_array_equal(again["variance"], out["variance"])


def test_alpha_cg_config5_recipe_cap(gpb_lib):
    """The prediction-time alpha solve on the config-5 recipe (RBF-ARD, d = 8,
    noise 0.01) at the reference's default settings (max 300 iterations,
    relative residual 1e-3; solve_single_rhs_deterministic_host_jit,
    jit_prediction.mojo:681-759: plain CG, no preconditioner). At n = 12000
    the float64 restatement of that algorithm also stops at the 300 cap, so
    a capped run at scale is the reference's behaviour, not this
    implementation's; the float32 solve reaches a residual of the same order
    (unconverged CG iterates themselves differ between float32 and float64)."""
    from mojogp_b200 import synthetic
    from oracle import kernels as ok
    n = 12000
    X, y, _, p, noise = synthetic.config5(n=n, n_test=1)
    k = make_ard_kernel(RBF(ard=True), 8)
    prov = Provider(X, k, p, noise)
    yc = (y - y.mean()).astype(np.float32)
    alpha, it = prediction.compute_alpha(prov, yc, 300, 1e-3)
    A = ok.kernel_matrix(k.to_spec(8), p, X) + noise * np.eye(n)
    b = yc.astype(np.float64)
    ref, rit = ol.alpha_cg(A, b, 300, 1e-3)
    assert rit == 300 and it == 300, (it, rit)
    res_gpu = np.linalg.norm(b - A @ alpha) / np.linalg.norm(b)
    res_ref = np.linalg.norm(b - A @ ref) / np.linalg.norm(b)
    assert res_ref > 1e-3 and res_gpu < 3 * res_ref, (res_gpu, res_ref)


def test_alpha_cg_config5_recipe_converged(gpb_lib):
    """Same recipe with noise 0.1 (better conditioned): both solves converge
    within the default budget and agree to the solve tolerance. float32 CG
    needs more iterations than float64 here (112 against 88 on this B200: the
    float32 residual recurrence loses orthogonality at condition ~1e4), so
    the counts are held to within 1.5x, not equal."""
    from mojogp_b200 import synthetic
    from oracle import kernels as ok
    n = 3000
    X, y, _, p, _ = synthetic.config5(n=n, n_test=1)
    noise = 0.1
    k = make_ard_kernel(RBF(ard=True), 8)
    prov = Provider(X, k, p, noise)
    yc = (y - y.mean()).astype(np.float32)
    alpha, it = prediction.compute_alpha(prov, yc, 300, 1e-3)
    A = ok.kernel_matrix(k.to_spec(8), p, X) + noise * np.eye(n)
    ref, rit = ol.alpha_cg(A, yc.astype(np.float64), 300, 1e-3)
    assert it < 300 and rit < 300 and rit <= it <= 1.5 * rit, (it, rit)
    assert np.linalg.norm(alpha - ref) / np.linalg.norm(ref) < 1e-2
