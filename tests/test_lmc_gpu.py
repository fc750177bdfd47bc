"""LMC operator, BBMM gradients and fit on the GPU vs the float64 oracle."""
import ctypes as C

import numpy as np
import pytest

from mojogp_b200 import synthetic
from mojogp_b200.kernel import RBF, Matern32, make_ard_kernel
from mojogp_b200.multi_output_gp import LMC, MultiOutputLMCGP
from mojogp_b200.provider import DeviceBuffer, Provider
from oracle import lmc as olmc

pytestmark = pytest.mark.gpu


def _setup(n=150, d=2, T=3, seed=0):
    rng = np.random.default_rng(seed)
    X = rng.uniform(-1, 1, size=(n, d)).astype(np.float32)
    ks = [RBF(), Matern32(), make_ard_kernel(RBF(ard=True), d)]
    ps = [np.array([0.5, 1.0], np.float32), np.array([0.6, 0.8], np.float32),
          np.array([0.7, 0.4, 1.1], np.float32)]
    # Condition number ~40 so a 30-iteration solve is converged in float32 and
    # float64 alike (at ~1e3 the unconverged float32 and float64 CG iterates
    # differ by more than the 1e-4 NLL bar; the float32 arithmetic is the
    # reference's own).
    A = np.stack([(lambda M: 0.1 * (M @ M.T) + 0.05 * np.eye(T))(rng.normal(size=(T, T)) * 0.5)
                  for _ in ks]).astype(np.float32)
    noise = rng.uniform(0.5, 1.0, size=T).astype(np.float32)
    provs = [Provider(X, k, p, 0.0) for k, p in zip(ks, ps)]
    lmc = LMC(provs, T)
    lmc.set_coregion(A, noise)
    return X, ks, ps, A, noise, provs, lmc


def test_lmc_matvec_vs_dense(gpb_lib):
    X, ks, ps, A, noise, provs, lmc = _setup()
    n, T, t = X.shape[0], A.shape[1], 5
    V = np.random.default_rng(1).standard_normal((t, T * n)).astype(np.float32)
    vd = DeviceBuffer.from_host(V)
    od = DeviceBuffer(V.shape)
    from mojogp_b200 import _lib
    _lib.call("gpb_lmc_matvec", C.c_void_p(lmc.handle), od.cptr, vd.cptr, t)
    K, _, _ = olmc.full_operator([k.to_spec(2) for k in ks], ps, X.astype(np.float64), A, noise)
    ref = (K @ V.T.astype(np.float64)).T
    got = od.download()
    assert np.linalg.norm(got - ref) / np.linalg.norm(ref) < 1e-5


def test_lmc_bbmm_vs_oracle(gpb_lib):
    X, ks, ps, A, noise, provs, lmc = _setup()
    rng = np.random.default_rng(2)
    Y = rng.standard_normal((X.shape[0], A.shape[1])).astype(np.float32)
    yc = (Y - Y.mean(0)).T.copy()
    got = lmc.bbmm(yc, 8, 30, 30, 0.0, 2, False)
    ref = olmc.lmc_bbmm([k.to_spec(2) for k in ks], ps, X, Y - Y.mean(0), A, noise, 8, 30, 30,
                        0.0, iteration=2)
    assert got["cg_iters"] == ref["cg_iters"]
    assert abs(got["nll"] - ref["nll"]) < 1e-4 * abs(ref["nll"])
    np.testing.assert_allclose(got["kgrads"], ref["kgrads"], rtol=0,
                               atol=1e-3 * np.abs(ref["kgrads"]).max())
    np.testing.assert_allclose(got["gA"], ref["gA"], rtol=0, atol=1e-3 * np.abs(ref["gA"]).max())
    np.testing.assert_allclose(got["gnoise"], ref["gnoise"], rtol=0,
                               atol=1e-3 * np.abs(ref["gnoise"]).max())
    np.testing.assert_allclose(got["sum_alpha"], ref["sum_alpha"], rtol=1e-3, atol=1e-3)


def test_lmc_fit_predict_config4_small(gpb_lib):
    X, Y = synthetic.config4(n=2000)
    gp = MultiOutputLMCGP(kernels=[RBF(), Matern32(), RBF(ard=True)], num_probes=10)
    gp.fit(X, Y, max_iterations=15, learning_rate=0.05)
    h = gp.nll_history
    assert np.all(np.isfinite(h)) and h[-1] < h[0]
    pred = gp.predict(X[:500])  # no flags: a MultiOutputPredictionResult, as the reference
    mean = pred.mean
    r2 = 1 - np.mean((mean - Y[:500]) ** 2) / np.var(Y[:500])
    assert mean.shape == (500, 4) and r2 > 0.8
    assert pred.variance.shape == (500, 4) and np.all(pred.variance > 0)
    np.testing.assert_allclose(pred.std, np.sqrt(pred.variance), rtol=1e-6)


def _ill_conditioned(n=150, d=2, T=3, seed=5):
    """Small task noise: the regime the LMC preconditioner exists for."""
    X, ks, ps, A, noise, provs, lmc = _setup(n, d, T, seed)
    noise = np.array([0.01, 0.02, 0.015][:T], np.float32)
    lmc.set_coregion(A, noise)
    return X, ks, ps, A, noise, provs, lmc


def test_lmc_precond_apply_logdet_sample_vs_oracle(gpb_lib):
    X, ks, ps, A, noise, provs, lmc = _ill_conditioned()
    n, T = X.shape[0], A.shape[1]
    ranks, logdet = lmc.build_precond(10)
    Ks = [olmc.ok.kernel_matrix(k.to_spec(2), p, X.astype(np.float64)) for k, p in zip(ks, ps)]
    # The greedy factor is float32 on the device as in the reference; at task
    # noise 0.01 its rounding-level trailing columns move log|P| by ~4 against a
    # float64 factor, so log|P| is pinned to the float32 factorisation.
    P = olmc.LmcPrecond(Ks, A, noise, 10, factor_dtype=np.float32)
    assert list(ranks) == P.ranks
    assert abs(logdet - P.logdet) < 1e-5 * abs(P.logdet)
    V = np.random.default_rng(3).standard_normal((6, T * n)).astype(np.float32)
    got = lmc.precond_apply_host(V)
    ref = P.apply(V.T.astype(np.float64)).T
    assert np.linalg.norm(got - ref) / np.linalg.norm(ref) < 1e-4
    Z = lmc.precond_sample_host(5, 77)
    Zr = P.sample(5, 77).T
    assert np.linalg.norm(Z - Zr) / np.linalg.norm(Zr) < 1e-4
    # rank <= 0 removes it
    r0, ld0 = lmc.build_precond(0)
    assert ld0 == 0.0 and not r0.any()


def test_lmc_bbmm_preconditioned_vs_oracle(gpb_lib):
    X, ks, ps, A, noise, provs, lmc = _ill_conditioned()
    rng = np.random.default_rng(4)
    Y = rng.standard_normal((X.shape[0], A.shape[1])).astype(np.float32)
    yc = (Y - Y.mean(0)).T.copy()
    plain = lmc.bbmm(yc, 8, 200, 30, 1e-2, 1, False)
    lmc.build_precond(15)
    got = lmc.bbmm(yc, 8, 200, 30, 1e-2, 1, False)
    ref = olmc.lmc_bbmm([k.to_spec(2) for k in ks], ps, X, Y - Y.mean(0), A, noise, 8, 200, 30,
                        1e-2, iteration=1, precond_rank=15)
    # The preconditioner cuts the iteration count of the same solve.
    assert got["cg_iters"] < plain["cg_iters"]
    assert abs(got["cg_iters"] - ref["cg_iters"]) <= 10
    assert abs(got["nll"] - ref["nll"]) < 1e-3 * abs(ref["nll"])
    np.testing.assert_allclose(got["gnoise"], ref["gnoise"], rtol=0,
                               atol=1e-2 * np.abs(ref["gnoise"]).max())
    np.testing.assert_allclose(got["gA"], ref["gA"], rtol=0, atol=1e-2 * np.abs(ref["gA"]).max())


def test_lmc_predict_variance_vs_exact_latents(gpb_lib):
    X, Y = synthetic.config4(n=600)
    gp = MultiOutputLMCGP(kernels=[RBF(), Matern32()], num_probes=8)
    gp.fit(X, Y, max_iterations=5, learning_rate=0.05)
    gp.lanczos_rank = 600  # LOVE rank = n: the root is exact up to float32
    Xt = X[:50]
    mean, var = gp.predict(Xt, return_var=True)
    _, std = gp.predict(Xt, return_std=True)
    np.testing.assert_allclose(std, np.sqrt(var), rtol=1e-6)
    # predict_lmc's formula with exact latent posteriors:
    avg = float(np.mean(gp.noise))
    Xd = X.astype(np.float64)
    ref = np.zeros_like(var, dtype=np.float64)
    for s, (k, p) in enumerate(zip(gp.kernels_resolved, gp.params_)):
        spec = k.to_spec(X.shape[1])
        K = olmc.ok.kernel_matrix(spec, p, Xd)
        Ks = olmc.ok.kernel_matrix(spec, p, Xd[:50], Xd)
        kss = np.diag(olmc.ok.kernel_matrix(spec, p, Xd[:50]))
        lat = kss - np.einsum("ij,ji->i", Ks, np.linalg.solve(K + avg * np.eye(len(X)), Ks.T))
        ref += np.maximum(lat, 1e-10)[:, None] * (gp.A[s] ** 2).sum(axis=1)[None, :]
    ref += gp.noise[None, :]
    assert var.shape == (50, 4)
    np.testing.assert_allclose(var, ref, rtol=2e-3, atol=1e-4)


def test_lmc_bbmm_rbf16_tensor_core_gradients(gpb_lib):
    """RBF-ARD latent at d = 16 takes the Gram K.V kernel and the tensor-core
    gradient reduction with T data columns; BBMM outputs against the oracle."""
    rng = np.random.default_rng(21)
    n, d, T = 400, 16, 3
    X = (0.6 * rng.standard_normal((n, d))).astype(np.float32)
    ks = [make_ard_kernel(RBF(ard=True), d), Matern32()]
    ps = [np.concatenate([rng.uniform(1.0, 2.0, d), [1.0]]).astype(np.float32),
          np.array([1.5, 0.7], np.float32)]
    A = np.stack([(lambda M: 0.1 * (M @ M.T) + 0.05 * np.eye(T))(rng.normal(size=(T, T)) * 0.5)
                  for _ in ks]).astype(np.float32)
    noise = rng.uniform(0.5, 1.0, size=T).astype(np.float32)
    provs = [Provider(X, k, p, 0.0) for k, p in zip(ks, ps)]
    assert provs[0].matvec_layout(16).startswith("gram-tensor-core")
    lmc = LMC(provs, T)
    lmc.set_coregion(A, noise)
    Y = rng.standard_normal((n, T)).astype(np.float32)
    yc = (Y - Y.mean(0)).T.copy()
    got = lmc.bbmm(yc, 8, 30, 30, 0.0, 2, False)
    ref = olmc.lmc_bbmm([k.to_spec(d) for k in ks], ps, X, Y - Y.mean(0), A, noise, 8, 30, 30,
                        0.0, iteration=2)
    assert abs(got["nll"] - ref["nll"]) < 1e-4 * abs(ref["nll"])
    for key in ("kgrads", "gA", "gnoise"):
        np.testing.assert_allclose(got[key], ref[key], rtol=0,
                                   atol=1e-3 * np.abs(ref[key]).max(), err_msg=key)


def _exact_var_ref(ks, ps, X, Xt, A, noise):
    return olmc.exact_variance([k.to_spec(X.shape[1]) for k in ks], ps, X.astype(np.float64),
                               Xt.astype(np.float64), A.astype(np.float64),
                               noise.astype(np.float64))


@pytest.mark.parametrize("block_cols", [0, 12])
def test_lmc_exact_variance_vs_oracle(gpb_lib, block_cols):
    X, ks, ps, A, noise, provs, lmc = _setup()
    Xt = np.random.default_rng(6).uniform(-1.2, 1.2, size=(37, X.shape[1])).astype(np.float32)
    # block_cols 12 at T = 3: blocks of 4 test points, the last one ragged (37 = 9 x 4 + 1).
    var, iters = lmc.exact_variance(Xt, 300, 1e-6, block_cols)
    ref = _exact_var_ref(ks, ps, X, Xt, A, noise)
    assert var.shape == (37, 3) and iters > 0
    np.testing.assert_allclose(var, ref, rtol=1e-3, atol=1e-5)
    # Posterior variance lies between the noise floor and the prior + noise.
    assert np.all(var >= noise[None, :] * (1 - 1e-4))


def test_lmc_exact_variance_preconditioned(gpb_lib):
    X, ks, ps, A, noise, provs, lmc = _ill_conditioned()
    Xt = np.random.default_rng(7).uniform(-1, 1, size=(20, X.shape[1])).astype(np.float32)
    ref = _exact_var_ref(ks, ps, X, Xt, A, noise)
    plain, it_plain = lmc.exact_variance(Xt, 1000, 1e-5)
    lmc.build_precond(15)
    pc, it_pc = lmc.exact_variance(Xt, 1000, 1e-5)
    assert it_pc < it_plain
    for v in (plain, pc):
        np.testing.assert_allclose(v, ref, rtol=2e-3, atol=2e-4)


def test_lmc_gp_predict_variance_methods(gpb_lib):
    X, Y = synthetic.config4(n=400)
    gp = MultiOutputLMCGP(kernels=[RBF(), Matern32()], num_probes=8, cg_tolerance=1e-4)
    gp.fit(X, Y, max_iterations=3, learning_rate=0.05)
    Xt = X[:30] + 0.05
    mean, var = gp.predict(Xt, return_var=True, variance_method="exact")
    _, std = gp.predict(Xt, return_std=True, variance_method="exact")
    np.testing.assert_allclose(std, np.sqrt(var), rtol=1e-5)
    ref = _exact_var_ref(gp.kernels_resolved, gp.params_, X, Xt, gp.A, gp.noise)
    np.testing.assert_allclose(var, ref, rtol=2e-3, atol=1e-4)
    m0, v0 = gp.predict(Xt, return_var=True, variance_method="mean_only")
    np.testing.assert_allclose(m0, mean)
    assert not v0.any()
    with pytest.raises(ValueError):
        gp.predict(Xt, return_var=True, variance_method="bogus")
