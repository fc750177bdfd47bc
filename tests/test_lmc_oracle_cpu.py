"""LMC and preconditioner oracles against dense float64 linear algebra (CPU):
the exact posterior variance against the joint-Gaussian conditional over
[train; test], and the Woodbury preconditioners against their dense forms."""
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


def test_pivoted_cholesky_woodbury_identities():
    """The oracle preconditioner (greedy pivoted Cholesky, Woodbury apply, log|P|)
    against dense linear algebra: P^{-1} V = solve(L L^T + s I, V) and
    log|P| = slogdet(L L^T + s I) (the identities the reference's
    tests/unit/test_matrix_operations.py:109-165 pins); pivots greedy on the
    residual diagonal with the lowest index on ties."""
    rng = np.random.default_rng(1)
    X = rng.uniform(-1, 1, size=(80, 2))
    K = ok.kernel_matrix(RBF().to_spec(2), np.array([0.6, 1.3]), X)
    from oracle import bbmm as ob
    P = ob.Precond(K, 0.05, 12)
    dense = P.L @ P.L.T + 0.05 * np.eye(80)
    V = rng.standard_normal((80, 4))
    np.testing.assert_allclose(P.apply(V), np.linalg.solve(dense, V), rtol=1e-9, atol=1e-9)
    assert abs(P.logdet - np.linalg.slogdet(dense)[1]) < 1e-9 * abs(P.logdet)
    # First pivot: all diagonals equal (stationary kernel) -> index 0.
    assert P.pivots[0] == 0 and len(set(P.pivots)) == len(P.pivots)
    # Residual diagonal after the factor is non-negative and below the start.
    resid = np.diag(K - P.L @ P.L.T)
    assert resid.min() > -1e-10 and resid.max() <= np.diag(K).max() + 1e-12


def test_lmc_preconditioner_dense_identities():
    """Sum-of-Kronecker Woodbury preconditioner of the LMC oracle against its
    dense form: apply and log|P|."""
    rng = np.random.default_rng(2)
    n, T = 30, 2
    X = rng.uniform(-1, 1, size=(n, 2))
    Ks = [ok.kernel_matrix(RBF().to_spec(2), np.array([0.5, 1.0]), X),
          ok.kernel_matrix(Matern32().to_spec(2), np.array([0.8, 0.7]), X)]
    A = np.stack([(lambda M: M @ M.T + 0.1 * np.eye(T))(rng.normal(size=(T, T))) for _ in Ks])
    noise = np.array([0.05, 0.08])
    P = olmc.LmcPrecond(Ks, A, noise, 6)
    D = P.dense()
    V = rng.standard_normal((n * T, 3))
    np.testing.assert_allclose(P.apply(V), np.linalg.solve(D, V), rtol=1e-8, atol=1e-8)
    assert abs(P.logdet - np.linalg.slogdet(D)[1]) < 1e-9 * abs(P.logdet)
