"""BBMM (mBCG + SLQ + gradients), preconditioner and the training loop on the
GPU against the float64 oracle restatement with identical probes.

Tolerances: NLL and CG solves within 1e-4 relative; gradients within 1e-3 of
their largest component (the stochastic trace terms are differences of
float32 CG solutions)."""
import ctypes as C

import numpy as np
import pytest

from mojogp_b200 import _lib, engine
from mojogp_b200.kernel import RBF, Matern52, make_ard_kernel
from mojogp_b200.provider import Provider
from oracle import bbmm as ob

pytestmark = pytest.mark.gpu


def test_hash_gaussian_bitwise_uniforms(gpb_lib):
    n = 100000
    out = np.zeros(n, np.float32)
    _lib.call("gpb_hash_gaussian", 0, C.c_void_p(out.ctypes.data), n, 104729 * 3 + 42)
    ref = ob.hash_gaussian(np.arange(n, dtype=np.uint64), 104729 * 3 + 42)
    np.testing.assert_allclose(out, ref, rtol=2e-6, atol=2e-6)


def _problem(kind, n=400, d=2, seed=0):
    rng = np.random.default_rng(seed)
    X = rng.uniform(0, 1, size=(n, d)).astype(np.float32)
    y = (np.sin(6 * X[:, 0]) + 0.1 * rng.standard_normal(n)).astype(np.float32)
    if kind == "rbf_ard":
        k = make_ard_kernel(RBF(ard=True), d)
        p = np.array([0.3] * d + [1.2], np.float32)
    else:
        k = Matern52()
        p = np.array([0.4, 0.9], np.float32)
    return X, y, k, p


@pytest.mark.parametrize("kind,rank", [("rbf_ard", 0), ("m52", 0), ("rbf_ard", 15), ("m52", 25)])
def test_bbmm_vs_oracle(gpb_lib, kind, rank):
    # A fixed CG budget (tolerance 0, 30 = max_tridiag iterations) so float32
    # and float64 runs take the same iterations; the convergence rule itself
    # is covered by test_bbmm_convergence_rule.
    X, y, k, p = _problem(kind)
    # Without a preconditioner keep K + noise I well conditioned: at condition
    # numbers ~1e4 float32 CG (as in the reference) and float64 CG part ways
    # after 30 iterations by more than the 1e-4 bar.
    noise = 0.05 if rank > 0 else 0.25
    yc = y - y.mean()
    prov = Provider(X, k, p, noise)
    got = engine.bbmm(prov, yc, num_probes=10, max_cg_iter=30, max_tridiag_iter=30, cg_tol=0.0,
                      precond_rank=rank, iteration=3)
    ref = ob.bbmm(k.to_spec(X.shape[1]), p, X, yc, noise, 10, 30, 30, 0.0, iteration=3,
                  precond_rank=rank)
    assert got["cg_iters"] == ref["cg_iters"] == 30
    assert abs(got["inv_quad"] - ref["inv_quad"]) < 1e-4 * abs(ref["inv_quad"])
    assert abs(got["logdet"] - ref["logdet"]) < 1e-4 * abs(ref["logdet"])
    assert abs(got["nll"] - ref["nll"]) < 1e-4 * abs(ref["nll"])
    g, rg = got["grads"], ref["grads"]
    np.testing.assert_allclose(g, rg, rtol=0, atol=1e-3 * np.abs(rg).max())


def test_bbmm_convergence_rule(gpb_lib):
    # Well-conditioned problem: both stop at the same check (every 10
    # iterations after 10, never before max_tridiag - 1).
    rng = np.random.default_rng(0)
    n, d = 400, 2
    X = rng.uniform(0, 1, size=(n, d)).astype(np.float32)
    y = (np.sin(6 * X[:, 0]) + 0.1 * rng.standard_normal(n)).astype(np.float32)
    k = make_ard_kernel(RBF(ard=True), d)
    p = np.array([0.5, 0.5, 1.0], np.float32)
    yc = y - y.mean()
    prov = Provider(X, k, p, 0.2)
    got = engine.bbmm(prov, yc, num_probes=10, max_cg_iter=100, max_tridiag_iter=30, cg_tol=1e-2,
                      precond_rank=0, iteration=1)
    ref = ob.bbmm(k.to_spec(d), p, X, yc, 0.2, 10, 100, 30, 1e-2, iteration=1)
    assert got["cg_iters"] == ref["cg_iters"]
    assert abs(got["nll"] - ref["nll"]) < 1e-4 * abs(ref["nll"])


def test_pivot_order_matches_oracle(gpb_lib):
    # Through gpb_bbmm with a preconditioner: identical log|P| requires the
    # same pivots; compare the preconditioner log-det contribution directly.
    X, y, k, p = _problem("rbf_ard", n=300)
    noise = 0.02
    prov = Provider(X, k, p, noise)
    yc = y - y.mean()
    g0 = engine.bbmm(prov, yc, num_probes=4, precond_rank=0, iteration=0)
    g1 = engine.bbmm(prov, yc, num_probes=4, precond_rank=30, iteration=0)
    from oracle import kernels as ok
    K = ok.kernel_matrix(k.to_spec(2), p, X)
    pc = ob.Precond(K, noise, 30)
    r1 = ob.bbmm(k.to_spec(2), p, X, yc, noise, 4, 100, 30, 1e-2, iteration=0, precond=pc)
    assert abs(g1["logdet"] - r1["logdet"]) < 1e-4 * abs(r1["logdet"])
    # the preconditioned and plain estimates describe the same log|K|
    assert abs(g1["logdet"] - g0["logdet"]) < 0.05 * abs(g0["logdet"])


def test_train_matches_oracle(gpb_lib):
    X, y, k, p = _problem("rbf_ard", n=300)
    noise = 0.3
    prov = Provider(X, k, p, noise)
    res = engine.train(prov, y, max_iterations=6, learning_rate=0.05, num_probes=10,
                       precond_rank=0, use_preconditioner=False, init_mean=float(y.mean()))
    ref = ob.train(k.to_spec(2), p, X, y, noise, max_iterations=6, learning_rate=0.05,
                   num_probes=10, precond_rank=0, init_mean=float(y.mean()))
    np.testing.assert_allclose(res["nll_history"], ref["nll_history"], rtol=1e-4)
    np.testing.assert_allclose(res["params"], ref["params"], rtol=1e-4)
    assert abs(res["noise"] - ref["noise"]) < 1e-4 * ref["noise"]
    assert abs(res["mean"] - ref["mean"]) < 1e-4 * max(1.0, abs(ref["mean"]))
    assert res["cached_alpha"] is not None


def test_train_with_preconditioner_runs(gpb_lib):
    X, y, k, p = _problem("m52", n=2000, d=3, seed=4)
    prov = Provider(X, k, p, 0.1)
    res = engine.train(prov, y, max_iterations=8, learning_rate=0.05, num_probes=10,
                       precond_rank=50, init_mean=float(y.mean()))
    h = res["nll_history"]
    assert np.all(np.isfinite(h)) and h[-1] < h[0]
    assert res["precond_rank"] == 50 and res["precond_build_count"] >= 1


def _pivot_check(prov, k, p, X, rank, tag):
    """GPU pivot list vs the oracle's greedy rule (float32 factor, as the
    reference's pivoted_cholesky.mojo). Pivots must be identical except at
    near-ties: steps where the oracle's own pick and the GPU's differ by less
    than 1e-6 of the residual diagonal. Those are listed in the failure text."""
    from oracle import kernels as ok
    got = engine.precond_pivots(prov, rank)
    spec = k.to_spec(X.shape[1])
    diag = np.array([ok.kernel_matrix(spec, p, X[i:i + 1])[0, 0] for i in range(1)])
    diag = np.full(X.shape[0], diag[0])  # stationary kernel: constant diagonal
    ref = ob.greedy_pivots(lambda i: ok.kernel_matrix(spec, p, X, X[i:i + 1])[:, 0], diag, rank,
                           follow=got["pivots"])
    gp = np.asarray(got["pivots"])
    assert len(gp) == len(ref["pivots"]) == rank, (tag, len(gp), len(ref["pivots"]))
    diff = np.nonzero(gp != np.asarray(ref["pivots"]))[0]
    ties = [(int(m), int(gp[m]), int(ref["pivots"][m]), float(ref["gap"][m])) for m in diff]
    assert all(g < 1e-6 for *_, g in ties), f"{tag}: pivots differ beyond near-ties: {ties}"
    np.testing.assert_allclose(got["values"], ref["followed_values"], rtol=1e-3, atol=1e-5)
    return ties


def test_pivot_indices_match_oracle_small(gpb_lib):
    X, y, k, p = _problem("rbf_ard", n=300)
    prov = Provider(X, k, p, 0.02)
    ties = _pivot_check(prov, k, p, X, 30, "rbf_ard n=300")
    assert not ties


def test_pivot_indices_match_oracle_config2_recipe(gpb_lib):
    # Config-2 recipe (Matern-5/2 ARD, d = 8, X ~ U[0,1]^8, rank 100) at n = 2e4.
    from mojogp_b200 import synthetic
    X, y = synthetic.config2(n=20_000)
    d = X.shape[1]
    k = make_ard_kernel(Matern52(ard=True), d)
    p = np.array([0.6, 0.8, 1.0, 0.7, 0.9, 1.1, 0.5, 0.75, 1.3], np.float32)
    prov = Provider(X, k, p, 0.01)
    ties = _pivot_check(prov, k, p, X, 100, "config2 n=2e4")
    assert len(ties) <= 2, ties


def test_pivot_index_exact_above_2_24(gpb_lib):
    # Indices beyond 2^24 are not exactly representable in float32; the GPU
    # keeps pivot indices as integers. X is a constant row except for one
    # row near the end whose kernel-row residual stays largest after step 0.
    n, d = (1 << 24) + 1000, 1
    X = np.zeros((n, d), np.float32)
    X[-3, 0] = 40.0    # far from every other row: picked second
    k = RBF()
    p = np.array([1.0, 1.0], np.float32)
    prov = Provider(X, k, p, 0.01)
    got = engine.precond_pivots(prov, 2)
    assert list(got["pivots"]) == [0, n - 3]
