"""Host numerics (no GPU): SLQ log-determinant and the tridiagonal
eigensolver, against the reference's own known-answer identities
(tests/unit/test_lanczos.py:212-245: SLQ on I gives 0, on c*I gives n log c)
and against numpy."""
import ctypes as C

import numpy as np
import pytest

from mojogp_b200 import _lib
from oracle import bbmm as ob


def _slq(diags, offs, n):
    diags = np.ascontiguousarray(diags, np.float64)
    offs = np.ascontiguousarray(offs, np.float64)
    out = C.c_double()
    p, m = diags.shape
    st = _lib.lib().gpb_slq_logdet(C.c_void_p(diags.ctypes.data), C.c_void_p(offs.ctypes.data), m,
                                   p, n, C.byref(out))
    assert st == 0
    return out.value


@pytest.mark.parametrize("c", [1.0, 2.5, 0.3])
def test_slq_scaled_identity_known_answer(gpb_lib, c):
    n, m, probes = 1000, 12, 5
    diags = np.full((probes, m), c)
    offs = np.zeros((probes, m - 1))
    assert abs(_slq(diags, offs, n) - n * np.log(c)) < 1e-9 * max(1, n * abs(np.log(c)))
    assert abs(ob.slq_logdet(list(diags), list(offs), n) - n * np.log(c)) < 1e-9 * max(1, n * abs(np.log(c)))


def test_slq_matches_oracle_random(gpb_lib):
    rng = np.random.default_rng(0)
    probes, m, n = 6, 20, 5000
    diags = rng.uniform(2, 5, size=(probes, m))
    offs = rng.uniform(0.1, 0.9, size=(probes, m - 1))
    got = _slq(diags, offs, n)
    ref = ob.slq_logdet(list(diags), list(offs), n)
    assert abs(got - ref) < 1e-9 * abs(ref)


def test_tridiag_eig_matches_numpy(gpb_lib):
    rng = np.random.default_rng(1)
    m = 40
    d = rng.normal(size=m)
    e = rng.normal(size=m - 1)
    ev = np.zeros(m)
    V = np.zeros((m, m))
    st = _lib.lib().gpb_tridiag_eig(C.c_void_p(d.ctypes.data), C.c_void_p(e.ctypes.data), m,
                                    C.c_void_p(ev.ctypes.data), C.c_void_p(V.ctypes.data))
    assert st == 0
    T = np.diag(d) + np.diag(e, 1) + np.diag(e, -1)
    np.testing.assert_allclose(ev, np.linalg.eigvalsh(T), atol=1e-10)
    np.testing.assert_allclose(T @ V, V * ev, atol=1e-9)
    np.testing.assert_allclose(V.T @ V, np.eye(m), atol=1e-10)


def test_hash_gaussian_oracle_statistics():
    z = ob.hash_gaussian(np.arange(200000, dtype=np.uint64), 42)
    assert abs(z.mean()) < 0.01 and abs(z.std() - 1) < 0.01
    # uniforms are exact integer arithmetic: u1 in (0,1], u2 in [0,1)
    z2 = ob.hash_gaussian(np.arange(10, dtype=np.uint64), 104729 + 42)
    assert np.all(np.isfinite(z2))
