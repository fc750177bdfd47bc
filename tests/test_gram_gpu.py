"""Gram-form tensor-core K·V path (both contractions on tcgen05) vs the fp64
oracle at the 1e-5 relative-Frobenius matvec bar, plus the host's choice of
path: taken for bounded prescaled norms and the leaves smooth in u at 0,
refused for Matérn-1/2, the composite evaluator and large norms (where the
difference-form kernels run and must still be exact to the same bar)."""
import numpy as np
import pytest

from mojogp_b200.kernel import RBF, RQ, Matern12, Matern32, Matern52, make_ard_kernel
from mojogp_b200.provider import DeviceBuffer, Provider
from oracle import kernels as ok
from tests.conftest import rel_fro

pytestmark = pytest.mark.gpu

LEAVES = {
    "rbf_ard": lambda d: make_ard_kernel(RBF(ard=True), d),
    "m32": lambda d: Matern32(),
    "m52_ard": lambda d: make_ard_kernel(Matern52(ard=True), d),
    "rq_ard": lambda d: make_ard_kernel(RQ(ard=True), d),
}


def _setup(kname, n, d, t, seed, ell=(0.5, 3.0), shift=0.0):
    rng = np.random.default_rng(seed)
    k = LEAVES[kname](d) if kname in LEAVES else kname
    kk = k.resolve_ard(d)
    names = kk.get_param_names()
    p = np.empty(kk.num_params(), np.float32)
    for i, nm in enumerate(names):
        p[i] = rng.uniform(*ell) if ("length" in nm or "_ls_" in nm) else rng.uniform(0.5, 2.0)
    X = (rng.standard_normal((n, d)) + shift).astype(np.float32)
    V = rng.standard_normal((n, t)).astype(np.float32)
    return k, p, X, V


@pytest.mark.parametrize("kname", sorted(LEAVES))
@pytest.mark.parametrize("n,d,t", [(5000, 16, 16), (1537, 16, 13), (700, 8, 16), (3000, 5, 32)])
def test_gram_matvec_vs_oracle(gpb_lib, kname, n, d, t):
    # Matérn prescaling multiplies by sqrt(3) or sqrt(5): longer lengthscales
    # keep those inputs inside the norm bound too.
    ell = (0.5, 3.0) if kname.startswith("rbf") or kname.startswith("rq") else (1.5, 3.0)
    k, p, X, V = _setup(kname, n, d, t, seed=n + d + t, ell=ell)
    prov = Provider(X, k, p, 0.1)
    assert prov.matvec_layout(t).startswith("gram-tensor-core")
    got = prov.matvec_host(V)
    ref = ok.forward_matvec(k.to_spec(d), p, X, V, noise=0.1)
    assert rel_fro(got, ref) < 1e-5


def test_gram_refused_for_large_norms(gpb_lib):
    # Shifted inputs with short lengthscales: max |x'|^2 far above the bound.
    k, p, X, V = _setup("rbf_ard", 2000, 16, 16, seed=5, ell=(0.5, 0.8), shift=3.0)
    prov = Provider(X, k, p, 0.1)
    assert prov.matvec_layout(16) == "tensor-core"
    ref = ok.forward_matvec(k.to_spec(16), p, X, V, noise=0.1)
    assert rel_fro(prov.matvec_host(V), ref) < 1e-5


@pytest.mark.parametrize("k", [Matern12(), RBF() + Matern52()])
def test_gram_refused_for_other_kernels(gpb_lib, k):
    rng = np.random.default_rng(2)
    d = 16
    X = rng.standard_normal((600, d)).astype(np.float32)
    p = rng.uniform(0.5, 2.0, size=k.resolve_ard(d).num_params()).astype(np.float32)
    prov = Provider(X, k, p, 0.1)
    assert not prov.matvec_layout(16).startswith("gram-tensor-core")


def test_gram_param_update_rechecks_bound(gpb_lib):
    # Shrinking the lengthscales raises the prescaled norms past the bound:
    # the next matvec must leave the Gram path and stay exact.
    k, p, X, V = _setup("rbf_ard", 1500, 16, 16, seed=9)
    prov = Provider(X, k, p, 0.1)
    assert prov.matvec_layout(16).startswith("gram-tensor-core")
    p2 = p.copy()
    names = k.resolve_ard(16).get_param_names()
    for i, nm in enumerate(names):
        if "length" in nm or "_ls_" in nm:
            p2[i] = 0.2
    prov.update_params(p2)
    assert prov.matvec_layout(16) == "tensor-core"
    ref = ok.forward_matvec(k.to_spec(16), p2, X, V, noise=0.1)
    assert rel_fro(prov.matvec_host(V), ref) < 1e-5


def test_gram_rows_and_cross(gpb_lib):
    # Row-sharded output rows use the Gram path; the cross matvec checks the
    # test rows' norms and takes the Gram path when they are bounded, the
    # difference form otherwise (shifted rows below). All against the oracle.
    k, p, X, V = _setup("rbf_ard", 2600, 16, 16, seed=4)
    prov = Provider(X, k, p, 0.1)
    full = prov.matvec_host(V)
    vd = DeviceBuffer.from_host(np.ascontiguousarray(V.T))
    od = DeviceBuffer((16, 1100))
    prov.forward_matvec_rows(od, vd, 16, 700, 1800)
    prov.synchronize()
    assert rel_fro(od.download().T, full[700:1800]) < 1e-6
    rng = np.random.default_rng(1)
    Xt = rng.standard_normal((333, 16)).astype(np.float32)
    got = prov.cross_matvec_host(Xt, V)
    ref = ok.cross_matvec(k.to_spec(16), p, Xt, X, V)
    assert rel_fro(got, ref) < 1e-5
    Xf = (Xt + 6.0).astype(np.float32)  # far outside the norm bound
    assert rel_fro(prov.cross_matvec_host(Xf, V), ok.cross_matvec(k.to_spec(16), p, Xf, X, V)) < 1e-5


@pytest.mark.parametrize("t", [1, 3, 8, 17])
@pytest.mark.parametrize("kname", ["rbf_ard", "m52_ard"])
def test_gram_narrow_blocks(gpb_lib, kname, t):
    # A single column (a Lanczos step, the alpha solve) runs on the narrow Gram
    # kernel; 2-15 columns on the Gram kernel with zero-padded columns; a
    # 17-column block is a 16-column chunk plus a 1-column narrow chunk.
    ell = (0.5, 3.0) if kname.startswith("rbf") else (1.5, 3.0)
    d = 16 if t in (3, 17) else 8
    k, p, X, V = _setup(kname, 2300, d, t, seed=30 + t, ell=ell)
    prov = Provider(X, k, p, 0.1)
    lay = prov.matvec_layout(t)
    assert lay == "gram-narrow" if t == 1 else lay.startswith("gram-tensor-core")
    ref = ok.forward_matvec(k.to_spec(d), p, X, V, noise=0.1)
    assert rel_fro(prov.matvec_host(V), ref) < 1e-5
    Xt = np.random.default_rng(t).standard_normal((101, d)).astype(np.float32)
    assert rel_fro(prov.cross_matvec_host(Xt, V), ok.cross_matvec(k.to_spec(d), p, Xt, X, V)) < 1e-5


@pytest.mark.parametrize("kname,n,d,t", [("rbf_ard", 3000, 16, 16), ("rbf_iso", 1000, 8, 11),
                                         ("rbf_ard", 777, 5, 20)])
def test_gram_gradient_bilinear_vs_oracle(gpb_lib, kname, n, d, t):
    """Tensor-core RBF gradient reduction (gradient_gram.cuh) against the
    float64 oracle: data column 0, probe columns 1.. (two chunks when t > 16)."""
    rng = np.random.default_rng(n + t)
    k = make_ard_kernel(RBF(ard=True), d) if kname == "rbf_ard" else RBF()
    kk = k.resolve_ard(d)
    p = np.array([rng.uniform(0.8, 2.0) for _ in range(kk.num_params())], np.float32)
    X = rng.standard_normal((n, d)).astype(np.float32)
    A = rng.standard_normal((n, t)).astype(np.float32)
    B = rng.standard_normal((n, t)).astype(np.float32)
    prov = Provider(X, k, p, 0.1)
    assert prov.matvec_layout(16).startswith("gram-tensor-core")
    ad = DeviceBuffer.from_host(np.ascontiguousarray(A.T))
    bd = DeviceBuffer.from_host(np.ascontiguousarray(B.T))
    data, trace = prov.gradient_bilinear(ad, bd, t)
    rd, rt = ok.gradient_bilinear(k.to_spec(d), p, X, A, B)
    np.testing.assert_allclose(data, rd, rtol=1e-4, atol=1e-4 * np.abs(rd).max())
    np.testing.assert_allclose(trace, rt, rtol=1e-4, atol=1e-4 * np.abs(rt).max())


def test_gram_fp16_column_scaling(gpb_lib):
    """The fp16 Gram path scales every right-hand-side column by a power of two
    from its own maximum: columns of very different magnitudes (and an all-zero
    column) in one product each meet the 1e-5 bar on their own."""
    k, p, X, _ = _setup("rbf_ard", 2500, 16, 16, seed=77)
    prov = Provider(X, k, p, 0.1)
    assert prov.matvec_layout(16).startswith("gram-tensor-core")
    rng = np.random.default_rng(78)
    mags = [1e-8, 1e-3, 1.0, 1e4, 1e8, 0.0, 3.0, 1e-20, 1e20, 1.0, 2.0, 5e-5, 7e6, 1.0, 1.0, 1.0]
    V = (rng.standard_normal((2500, 16)) * np.asarray(mags)[None, :]).astype(np.float32)
    got = prov.matvec_host(V)
    ref = ok.forward_matvec(k.to_spec(16), p, X, V, noise=0.1)
    for c, m in enumerate(mags):
        if m == 0.0:
            assert np.all(got[:, c] == 0.0)
        else:
            assert rel_fro(got[:, c], ref[:, c]) < 1e-5, (c, m)
