"""Gram-form tensor-core path at the inputs the headline benchmark runs on,
and just under the norm gate that admits the path.

The Gram expansion u = |x|^2 + |y|^2 - 2 x.y loses absolute accuracy in
proportion to the prescaled squared norms max |x'|^2; the host admits the path
up to kGramMaxSqNorm = 100 (csrc/kv_launch.cuh). These tests hold the matvec to
the 1e-5 relative-Frobenius bar and the fused RBF gradient reduction
(gb_kernel) to 1e-4 against the float64 oracle
(oracle/kernels.py, restating codegen_engine/expressions.py:77-240 and
passes/numerical_stability.py:13-112):

* the exact config-3 inputs (n = 1e6, d = 16, X ~ N(0, I), l ~ U[0.5, 3],
  seed 3): the full 16-column K.V on the GPU, checked on the 256 rows with the
  largest |x'|^2 plus 256 random rows, each over all 1e6 columns;
* synthetic inputs rescaled so that max |x'|^2 = 95, for RBF, Matern-3/2,
  Matern-5/2 and RQ;
* gb_kernel on a 3000-row subsample of config 3 (the 1500 largest-norm rows
  plus 1500 random ones) and on the max |x'|^2 = 95 inputs.
"""
import concurrent.futures as cf
import os

import numpy as np
import pytest

from mojogp_b200 import synthetic
from mojogp_b200.kernel import RBF, RQ, Matern32, Matern52, make_ard_kernel
from mojogp_b200.provider import DeviceBuffer, Provider
from oracle import kernels as ok
from tests.conftest import rel_fro

pytestmark = pytest.mark.gpu

# Square of the constant the provider folds into the prescaled inputs
# (x' = x * c / l): RBF log2(e)/2, Matern-nu 2 nu, RQ 1.
C2 = {"rbf": 0.5 / np.log(2.0), "m32": 3.0, "m52": 5.0, "rq": 1.0}
CTOR = {"rbf": RBF, "m32": Matern32, "m52": Matern52, "rq": RQ}


def _sqnorm(X, ell, kname):
    return C2[kname] * (((X.astype(np.float64)) / ell) ** 2).sum(axis=1)


def _params(k, d, ell, rng):
    names = k.resolve_ard(d).get_param_names()
    p, q = [], 0
    for nm in names:
        if "length" in nm or "_ls_" in nm:
            p.append(ell[q])
            q += 1
        else:
            p.append(rng.uniform(0.8, 1.5))
    return np.asarray(p, np.float32)


def test_config3_row_sample_vs_oracle(gpb_lib):
    X, _, ell = synthetic.config3()
    n, d, t = X.shape[0], X.shape[1], 16
    k = make_ard_kernel(RBF(ard=True), d)
    p = np.concatenate([ell, [1.0]]).astype(np.float32)
    sq = _sqnorm(X, ell, "rbf")
    assert 50.0 < sq.max() < 100.0  # the operating point (57.9 at seed 3)
    prov = Provider(X, k, p, 0.0025)
    assert prov.matvec_layout(t).startswith("gram-tensor-core")
    V = np.random.default_rng(7).standard_normal((t, n)).astype(np.float32)  # [t][n]
    vd = DeviceBuffer.from_host(np.ascontiguousarray(V))
    od = DeviceBuffer((t, n))
    prov.forward_matvec(od, vd, t)
    prov.synchronize()
    got = od.download()
    rng = np.random.default_rng(11)
    top = np.argsort(sq)[-256:]
    rnd = rng.choice(n, 256, replace=False)
    spec, Vt = k.to_spec(d), np.ascontiguousarray(V.T)

    def oracle_rows(r):  # numpy releases the GIL: row blocks run on all host cores
        return ok.forward_matvec(spec, p, X, Vt, noise=0.0025, rows=r, block=len(r))

    workers = min(8, os.cpu_count() or 1)
    for name, rows in (("largest |x'|^2", np.sort(top)), ("random", np.sort(rnd))):
        with cf.ThreadPoolExecutor(workers) as ex:
            ref = np.concatenate(list(ex.map(oracle_rows, np.array_split(rows, 16))))
        err = rel_fro(got[:, rows].T, ref)
        assert err < 1e-5, f"{name} rows: {err:.3e}"


def _near_gate_inputs(kname, n=6000, d=16, target=95.0, seed=0):
    rng = np.random.default_rng(seed)
    X = rng.standard_normal((n, d))
    ell = rng.uniform(0.8, 3.0, size=d)
    X *= np.sqrt(target / _sqnorm(X, ell, kname).max())
    X = X.astype(np.float32)
    assert 90.0 < _sqnorm(X, ell, kname).max() <= 95.5
    return X, ell.astype(np.float32), rng


@pytest.mark.parametrize("kname", ["rbf", "m32", "m52", "rq"])
def test_near_gate_matvec_vs_oracle(gpb_lib, kname):
    d, t = 16, 16
    X, ell, rng = _near_gate_inputs(kname, seed=len(kname))
    k = make_ard_kernel(CTOR[kname](ard=True), d)
    p = _params(k, d, ell, rng)
    prov = Provider(X, k, p, 0.01)
    assert prov.matvec_layout(t).startswith("gram-tensor-core")
    V = rng.standard_normal((X.shape[0], t)).astype(np.float32)
    ref = ok.forward_matvec(k.to_spec(d), p, X, V, noise=0.01)
    err = rel_fro(prov.matvec_host(V), ref)
    assert err < 1e-5, f"{kname}: {err:.3e}"
    # The one-column narrow Gram kernel (Lanczos and alpha steps) at the same inputs.
    assert prov.matvec_layout(1) == "gram-narrow"
    err1 = rel_fro(prov.matvec_host(V[:, :1]), ref[:, :1])
    assert err1 < 1e-5, f"{kname} narrow: {err1:.3e}"


def _check_bilinear(X, k, p, d, rng):
    n, t = X.shape[0], 16
    prov = Provider(X, k, p, 0.01)
    assert prov.matvec_layout(16).startswith("gram-tensor-core")
    A = rng.standard_normal((n, t)).astype(np.float32)
    B = rng.standard_normal((n, t)).astype(np.float32)
    ad = DeviceBuffer.from_host(np.ascontiguousarray(A.T))
    bd = DeviceBuffer.from_host(np.ascontiguousarray(B.T))
    data, trace = prov.gradient_bilinear(ad, bd, t)
    rd, rt = ok.gradient_bilinear(k.to_spec(d), p, X, A, B)
    np.testing.assert_allclose(data, rd, rtol=1e-4, atol=1e-4 * np.abs(rd).max())
    np.testing.assert_allclose(trace, rt, rtol=1e-4, atol=1e-4 * np.abs(rt).max())


def test_gb_kernel_config3_subsample(gpb_lib):
    X, _, ell = synthetic.config3()
    sq = _sqnorm(X, ell, "rbf")
    rng = np.random.default_rng(12)
    top = np.argsort(sq)[-1500:]
    rest = np.setdiff1d(np.arange(X.shape[0]), top)
    rows = np.concatenate([top, rng.choice(rest, 1500, replace=False)])
    Xs = np.ascontiguousarray(X[rows])
    d = X.shape[1]
    k = make_ard_kernel(RBF(ard=True), d)
    p = np.concatenate([ell, [1.0]]).astype(np.float32)
    _check_bilinear(Xs, k, p, d, rng)


def test_gb_kernel_near_gate(gpb_lib):
    X, ell, rng = _near_gate_inputs("rbf", n=3000, seed=5)
    d = X.shape[1]
    k = make_ard_kernel(RBF(ard=True), d)
    p = _params(k, d, ell, rng)
    _check_bilinear(X, k, p, d, rng)


def test_gb_kernel_config3_full_columns(gpb_lib):
    """The fused RBF gradient reduction over all 1e6 columns of config 3
    (every row's sum runs the full column range, where an unwindowed
    tensor-core accumulator would drift), with A zero outside 32 rows (the
    16 largest |x'|^2 and 16 random) so the float64 oracle can follow it."""
    X, _, ell = synthetic.config3()
    n, d, t = X.shape[0], X.shape[1], 16
    sq = _sqnorm(X, ell, "rbf")
    rng = np.random.default_rng(13)
    rows = np.unique(np.concatenate([np.argsort(sq)[-16:], rng.choice(n, 16, replace=False)]))
    k = make_ard_kernel(RBF(ard=True), d)
    p = np.concatenate([ell, [1.0]]).astype(np.float32)
    prov = Provider(X, k, p, 0.0025)
    assert prov.matvec_layout(16).startswith("gram-tensor-core")
    A = np.zeros((t, n), np.float32)
    A[:, rows] = rng.standard_normal((t, len(rows))).astype(np.float32)
    B = rng.standard_normal((t, n)).astype(np.float32)
    ad, bd = DeviceBuffer.from_host(A), DeviceBuffer.from_host(B)
    data, trace = prov.gradient_bilinear(ad, bd, t)
    spec = k.to_spec(d)

    def part(r):
        return ok.gradient_bilinear_rows(spec, p, X, r, A[:, r].T, B.T, block=2)

    with cf.ThreadPoolExecutor(min(8, os.cpu_count() or 1)) as ex:
        parts = list(ex.map(part, np.array_split(rows, 8)))
    rd = sum(q[0] for q in parts)
    rt = sum(q[1] for q in parts)
    np.testing.assert_allclose(data, rd, rtol=1e-4, atol=1e-4 * np.abs(rd).max())
    np.testing.assert_allclose(trace, rt, rtol=1e-4, atol=1e-4 * np.abs(rt).max())
