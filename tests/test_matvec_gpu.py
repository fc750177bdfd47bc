"""K·V, cross, diagonal, kernel-column and gradient kernels vs the fp64 oracle.

Tolerance: matvec outputs within 1e-5 relative Frobenius of the float64
oracle (the stated bar for this path); gradient reductions within 1e-4.
"""
import numpy as np
import pytest

from mojogp_b200.kernel import (RBF, RQ, Linear, Matern12, Matern32, Matern52, Periodic,
                                Polynomial, make_ard_kernel)
from mojogp_b200.provider import DeviceBuffer, Provider
from oracle import kernels as ok
from tests.conftest import rel_fro

pytestmark = pytest.mark.gpu

KERNELS = {
    "rbf": lambda d: RBF(),
    "rbf_ard": lambda d: make_ard_kernel(RBF(ard=True), d),
    "m12": lambda d: Matern12(),
    "m12_ard": lambda d: make_ard_kernel(Matern12(ard=True), d),
    "m32": lambda d: Matern32(),
    "m52_ard": lambda d: make_ard_kernel(Matern52(ard=True), d),
    "rq": lambda d: RQ(),
    "rq_ard": lambda d: make_ard_kernel(RQ(ard=True), d),
    "periodic": lambda d: Periodic(),
    "linear": lambda d: Linear(),
    "poly": lambda d: Polynomial(degree=2),
    "sum": lambda d: RBF() + Matern52(),
    "product": lambda d: RBF() * Linear(),
    "scale": lambda d: 2.0 * RBF(),
    "active": lambda d: RBF(active_dims=[0]) + Matern32(active_dims=list(range(1, d))),
}


def _params(k, d, rng):
    kk = k.resolve_ard(d)
    p = rng.uniform(0.5, 2.0, size=kk.num_params()).astype(np.float32)
    names = kk.get_param_names()
    for i, nm in enumerate(names):
        if "linear" in nm or "polynomial" in nm:
            p[i] = rng.uniform(0.2, 0.6)
        if nm.endswith("degree"):
            p[i] = 2.0
    return kk, p


@pytest.mark.parametrize("kname", sorted(KERNELS))
@pytest.mark.parametrize("n,d,t", [(300, 3, 11), (129, 2, 1), (1000, 8, 16)])
def test_forward_matvec_vs_oracle(gpb_lib, kname, n, d, t):
    rng = np.random.default_rng(7)
    if kname == "active" and d < 2:
        pytest.skip("needs d >= 2")
    k, p = _params(KERNELS[kname](d), d, rng)
    X = rng.uniform(0, 1, size=(n, d)).astype(np.float32)
    V = rng.standard_normal((n, t)).astype(np.float32)
    prov = Provider(X, k, p, 0.1)
    got = prov.matvec_host(V)
    ref = ok.forward_matvec(k.to_spec(d), p, X, V, noise=0.1)
    assert rel_fro(got, ref) < 1e-5


@pytest.mark.parametrize("n", [1, 2, 127, 128, 129, 255, 257, 4099])
@pytest.mark.parametrize("t", [1, 3, 4, 5, 16, 17, 33])
def test_forward_edges(gpb_lib, n, t):
    rng = np.random.default_rng(n * 100 + t)
    d = 5
    k = make_ard_kernel(RBF(ard=True), d)
    p = rng.uniform(0.5, 2.0, size=d + 1).astype(np.float32)
    X = rng.standard_normal((n, d)).astype(np.float32)
    V = rng.standard_normal((n, t)).astype(np.float32)
    prov = Provider(X, k, p, 0.05)
    got = prov.matvec_host(V)
    ref = ok.forward_matvec(k.to_spec(d), p, X, V, noise=0.05)
    assert got.shape == (n, t)
    assert rel_fro(got, ref) < 1e-5


@pytest.mark.parametrize("d", [1, 2, 3, 16, 17, 32])
def test_forward_dims(gpb_lib, d):
    rng = np.random.default_rng(d)
    n, t = 700, 16
    k = make_ard_kernel(RBF(ard=True), d)
    p = rng.uniform(0.5, 3.0, size=d + 1).astype(np.float32)
    X = rng.standard_normal((n, d)).astype(np.float32)
    V = rng.standard_normal((n, t)).astype(np.float32)
    prov = Provider(X, k, p, 0.1)
    assert rel_fro(prov.matvec_host(V), ok.forward_matvec(k.to_spec(d), p, X, V, noise=0.1)) < 1e-5


def test_fixed_noise_vector(gpb_lib):
    rng = np.random.default_rng(3)
    n, d, t = 500, 4, 8
    k = Matern52()
    p = np.array([0.7, 1.3], np.float32)
    X = rng.uniform(size=(n, d)).astype(np.float32)
    V = rng.standard_normal((n, t)).astype(np.float32)
    nv = rng.uniform(0.01, 0.3, size=n).astype(np.float32)
    prov = Provider(X, k, p, 0.0, noise_vector=nv)
    ref = ok.forward_matvec(k.to_spec(d), p, X, V, noise_vec=nv)
    assert rel_fro(prov.matvec_host(V), ref) < 1e-5


def test_row_sharded_matvec_concatenates(gpb_lib):
    rng = np.random.default_rng(11)
    n, d, t = 3000, 16, 16
    k = make_ard_kernel(RBF(ard=True), d)
    p = rng.uniform(0.5, 3, size=d + 1).astype(np.float32)
    X = rng.standard_normal((n, d)).astype(np.float32)
    V = rng.standard_normal((n, t)).astype(np.float32)
    prov = Provider(X, k, p, 0.1)
    full = prov.matvec_host(V)
    vd = DeviceBuffer.from_host(np.ascontiguousarray(V.T))
    parts = []
    bounds = [0, 700, 1500, 3000]
    for r0, r1 in zip(bounds[:-1], bounds[1:]):
        od = DeviceBuffer((t, r1 - r0))
        prov.forward_matvec_rows(od, vd, t, r0, r1)
        prov.synchronize()
        parts.append(od.download().T)
    np.testing.assert_allclose(np.concatenate(parts), full, rtol=0, atol=1e-5 * np.abs(full).max())


@pytest.mark.parametrize("kname", ["rbf_ard", "m52_ard", "sum", "periodic"])
def test_cross_diag_column(gpb_lib, kname):
    rng = np.random.default_rng(5)
    n, nt, d, t = 800, 333, 3, 7
    k, p = _params(KERNELS[kname](d), d, rng)
    X = rng.uniform(size=(n, d)).astype(np.float32)
    Xt = rng.uniform(-0.2, 1.2, size=(nt, d)).astype(np.float32)
    V = rng.standard_normal((n, t)).astype(np.float32)
    prov = Provider(X, k, p, 0.1)
    spec = k.to_spec(d)
    assert rel_fro(prov.cross_matvec_host(Xt, V), ok.cross_matvec(spec, p, Xt, X, V)) < 1e-5
    dd = DeviceBuffer(n)
    prov.extract_diagonal(dd)
    prov.synchronize()
    np.testing.assert_allclose(dd.download(), np.diag(ok.kernel_matrix(spec, p, X)), rtol=1e-5)
    col = DeviceBuffer(n)
    prov.kernel_column(col, 17)
    prov.synchronize()
    np.testing.assert_allclose(col.download(), ok.kernel_matrix(spec, p, X, X[17:18])[:, 0],
                               rtol=1e-5, atol=1e-7)


@pytest.mark.parametrize("kname", ["rbf", "rbf_ard", "m12_ard", "m32", "m52_ard", "rq_ard",
                                   "scale", "sum", "product", "periodic", "poly"])
def test_gradient_bilinear_vs_oracle(gpb_lib, kname):
    rng = np.random.default_rng(9)
    n, d, t = 600, 3, 11
    k, p = _params(KERNELS[kname](d), d, rng)
    X = rng.uniform(size=(n, d)).astype(np.float32)
    A = rng.standard_normal((n, t)).astype(np.float32)
    B = rng.standard_normal((n, t)).astype(np.float32)
    prov = Provider(X, k, p, 0.1)
    ad = DeviceBuffer.from_host(np.ascontiguousarray(A.T))
    bd = DeviceBuffer.from_host(np.ascontiguousarray(B.T))
    data, trace = prov.gradient_bilinear(ad, bd, t)
    rd, rt = ok.gradient_bilinear(k.to_spec(d), p, X, A, B)
    mask = k.engine_trainable_mask()
    scale_d = np.abs(rd).max()
    scale_t = np.abs(rt).max()
    np.testing.assert_allclose(data[mask], rd[mask], rtol=1e-4, atol=1e-4 * scale_d)
    np.testing.assert_allclose(trace[mask], rt[mask], rtol=1e-4, atol=1e-4 * scale_t)


def test_gradient_matvec_reference_layout(gpb_lib):
    rng = np.random.default_rng(13)
    n, d, t = 200, 2, 3
    k = make_ard_kernel(Matern52(ard=True), d)
    p = rng.uniform(0.5, 2, size=d + 1).astype(np.float32)
    X = rng.uniform(size=(n, d)).astype(np.float32)
    V = rng.standard_normal((n, t)).astype(np.float32)
    prov = Provider(X, k, p, 0.1)
    vd = DeviceBuffer.from_host(np.ascontiguousarray(V.T))
    od = DeviceBuffer((d + 1, t, n))
    prov.fused_gradient_matvec(od, vd, t)
    prov.synchronize()
    got = od.download()
    _, G = ok.kernel_matrix(k.to_spec(d), p, X, want_grad=True)
    for q in range(d + 1):
        assert rel_fro(got[q].T, G[q] @ V) < 1e-5
    od1 = DeviceBuffer((t, n))
    prov.gradient_matvec(od1, vd, t, 1)
    prov.synchronize()
    assert rel_fro(od1.download().T, G[1] @ V) < 1e-5


def test_host_matvec_from_pinned_buffers(gpb_lib):
    """gpb_forward_matvec_host reads and writes page-locked host buffers
    (gpb_host_register) with the same result as pageable ones, and the
    buffers stay usable after unregistering."""
    import ctypes as C

    from mojogp_b200 import _lib
    from mojogp_b200.provider import pinned

    rng = np.random.default_rng(31)
    n, d, t = 3000, 16, 16
    X = rng.standard_normal((n, d)).astype(np.float32)
    k = make_ard_kernel(RBF(ard=True), d)
    p = rng.uniform(0.8, 3.0, size=d + 1).astype(np.float32)
    prov = Provider(X, k, p, 0.01)
    Vc = np.ascontiguousarray(rng.standard_normal((t, n)).astype(np.float32))
    ref = prov.matvec_host(Vc.T)
    out = np.empty_like(Vc)
    with pinned(Vc, out):
        for _ in range(2):
            out[:] = 0
            _lib.call("gpb_forward_matvec_host", prov.h, C.c_void_p(out.ctypes.data),
                      C.c_void_p(Vc.ctypes.data), t)
            assert rel_fro(out.T, ref) < 1e-6
    assert rel_fro(out.T, ok.forward_matvec(k.to_spec(d), p, X, Vc.T, noise=0.01)) < 1e-5
