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
    mean = gp.predict(X[:500])
    r2 = 1 - np.mean((mean - Y[:500]) ** 2) / np.var(Y[:500])
    assert mean.shape == (500, 4) and r2 > 0.8
