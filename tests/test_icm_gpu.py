"""MultiOutputGP (ICM) on the LMC engine: the operator is the one-latent LMC
with A = os * B (checked against the dense float64 operator), a fit reduces the
NLL and predicts held-out tasks, and the predictive variance follows the
reference's eigen-route formula (checked densely with LOVE rank = n)."""
import numpy as np
import pytest

from mojogp_b200.kernel import RBF, Matern52
from mojogp_b200.multi_output_gp import MultiOutputGP, _icm_initial_W
from oracle import kernels as ok


def _data(n=500, T=3, seed=0):
    rng = np.random.default_rng(seed)
    X = rng.uniform(-1, 1, size=(n, 2)).astype(np.float32)
    f = np.sin(3 * X[:, 0]) + 0.5 * np.cos(2 * X[:, 1])
    g = np.cos(4 * X[:, 1])
    W = np.array([[1.0, 0.2], [0.8, -0.5], [0.3, 1.0]])[:T]
    Y = (np.stack([f, g], 1) @ W.T + 0.05 * rng.standard_normal((n, T))).astype(np.float32)
    return X, Y


def test_icm_initial_W_range():
    W = _icm_initial_W(4, 2)
    assert W.shape == (4, 2) and np.all(W >= 0.1) and np.all(W <= 0.5)
    assert np.array_equal(W, _icm_initial_W(4, 2))


@pytest.mark.gpu
def test_icm_fit_predict(gpb_lib):
    X, Y = _data()
    gp = MultiOutputGP(kernel="rbf", num_probes=8)
    gp.fit(X, Y, max_iterations=25, learning_rate=0.05)
    h = gp.nll_history
    assert np.all(np.isfinite(h)) and h.min() < h[0]
    pred = gp.predict(X[:200])  # no flags: a MultiOutputPredictionResult, as the reference
    mean = pred.mean
    assert pred.variance.shape == (200, 3) and np.all(np.isfinite(pred.std))
    r2 = 1 - np.mean((mean - Y[:200]) ** 2) / np.var(Y[:200])
    assert mean.shape == (200, 3) and r2 > 0.9
    B = gp.task_covariance
    assert np.allclose(B, B.T) and np.all(np.linalg.eigvalsh(B) > 0)


@pytest.mark.gpu
def test_icm_variance_matches_eigen_formula(gpb_lib):
    X, Y = _data(n=300)
    gp = MultiOutputGP(kernel=Matern52(), num_probes=6)
    gp.fit(X, Y, max_iterations=4)
    Xt = X[:40]
    _, var = gp.predict(Xt, return_var=True, lanczos_rank=300)
    _, var_x = gp.predict(Xt, return_var=True, variance_method="exact")
    spec = gp.kernel_resolved.to_spec(2)
    Xd = X.astype(np.float64)
    K = ok.kernel_matrix(spec, gp.params_, Xd)
    Ks = ok.kernel_matrix(spec, gp.params_, Xd[:40], Xd)
    kss = np.diag(ok.kernel_matrix(spec, gp.params_, Xd[:40]))
    ev, Q = np.linalg.eigh(gp.task_covariance)
    ev = np.maximum(ev, 1e-6)
    s2 = float(np.mean(gp.noise_per_task))
    ref = np.zeros((40, 3))
    for s in range(3):
        nz = s2 / ev[s]
        lat = kss - np.einsum("ij,ji->i", Ks, np.linalg.solve(K + nz * np.eye(len(X)), Ks.T))
        ref += (Q[:, s] ** 2 * ev[s])[None, :] * np.maximum(lat, 1e-10)[:, None]
    np.testing.assert_allclose(var, ref, rtol=5e-3, atol=1e-5)
    np.testing.assert_allclose(var_x, ref, rtol=2e-2, atol=1e-4)


def test_icm_initial_W_matches_oracle():
    from oracle import icm as oi
    np.testing.assert_array_equal(_icm_initial_W(5, 3), oi.initial_W(5, 3))


@pytest.mark.gpu
@pytest.mark.parametrize("kernel,R", [("rbf", -1), ("matern52", 2)])
def test_icm_fit_matches_oracle(gpb_lib, kernel, R):
    """Five iterations of the ICM fit against the float64 restatement of
    train_multi_output_jit (oracle/icm.py), both at the default CG tolerance
    1e-2 with no preconditioner and a well-conditioned start (noise 1.0), so
    the float32 and float64 mBCG runs take the same iteration counts; the
    probes are the library's counter-hash Gaussians on both sides.

    Bars: NLL history 1e-4 relative; the best state's kernel parameters,
    outputscale, noise, means, W and os * B within 3e-4 of each block's
    largest entry. The parameter bar is looser than the NLL bar because of
    float32 CG: after 30 iterations the float32 recursive residual stalls
    near 5e-5 where float64 reaches 2e-6, so the solves (and the stochastic
    gradients) differ by ~1e-4 relative, and Adam, which divides each
    gradient by its running RMS, turns that into step differences of about
    lr x 1e-3 that add up over the iterations."""
    from oracle import icm as oi
    X, Y = _data(n=300, T=3, seed=1)
    gp = MultiOutputGP(kernel=kernel, task_rank=R, num_probes=8, use_preconditioner=False)
    gp.fit(X, Y, max_iterations=5, learning_rate=0.05, initial_noise=1.0)
    spec = gp.kernel_resolved.to_spec(2)
    p0 = np.asarray(gp.kernel_resolved.get_initial_params(), np.float64)
    ref = oi.icm_fit(spec, X, Y, p0, max_iterations=5, learning_rate=0.05, task_rank=R,
                     num_probes=8, max_cg=200, cg_tol=1e-2, precond_rank=0, initial_noise=1.0,
                     trainable=gp.kernel_resolved.engine_trainable_mask())
    assert list(gp.cg_iterations_history) == list(ref["cg_iterations"])
    np.testing.assert_allclose(gp.nll_history, ref["nll_history"], rtol=1e-4)

    def close(a, b, what):
        a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
        assert np.max(np.abs(a - b)) <= 3e-4 * max(np.max(np.abs(b)), 1e-12), (what, a, b)

    close(gp.params_, ref["params"], "kernel params")
    close(gp.outputscale_, ref["outputscale"], "outputscale")
    close(gp.noise_per_task, ref["noise"], "noise")
    close(gp.mean_, ref["mean"], "means")
    close(gp.W_, ref["W"], "W")
    close(gp.task_covariance, ref["outputscale"] * ref["B"], "os * B")
