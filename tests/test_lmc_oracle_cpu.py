"""The LMC oracle's exact posterior variance against the textbook joint-Gaussian
conditional over [train; test] (CPU, float64)."""
import numpy as np

from mojogp_b200.kernel import RBF, Matern32
from oracle import kernels as ok
from oracle import lmc as olmc


def test_lmc_exact_variance_matches_joint_conditional():
    rng = np.random.default_rng(0)
    n, m, d, T = 40, 7, 2, 3
    X = rng.uniform(-1, 1, size=(n, d))
    Xt = rng.uniform(-1, 1, size=(m, d))
    specs = [RBF().to_spec(d), Matern32().to_spec(d)]
    ps = [np.array([0.5, 1.0]), np.array([0.7, 0.6])]
    A = np.stack([(lambda M: M @ M.T + 0.1 * np.eye(T))(rng.normal(size=(T, T))) for _ in specs])
    noise = rng.uniform(0.1, 0.3, size=T)
    got = olmc.exact_variance(specs, ps, X, Xt, A, noise)
    # Joint prior over all n + m points, task-blocked: sum_s A_s (x) K_s([X; X*]).
    Z = np.vstack([X, Xt])
    N = n + m
    J = sum(np.kron(A[s], ok.kernel_matrix(specs[s], ps[s], Z)) for s in range(len(specs)))
    tr = np.concatenate([np.arange(t * N, t * N + n) for t in range(T)])
    te = np.concatenate([np.arange(t * N + n, (t + 1) * N) for t in range(T)])
    Kxx = J[np.ix_(tr, tr)] + np.kron(np.diag(noise), np.eye(n))
    post = J[np.ix_(te, te)] - J[np.ix_(te, tr)] @ np.linalg.solve(Kxx, J[np.ix_(tr, te)])
    ref = np.diag(post).reshape(T, m).T + noise[None, :]
    np.testing.assert_allclose(got, ref, rtol=1e-10, atol=1e-12)
