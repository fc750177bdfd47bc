"""The no-allocation forward matvec (gpb_forward_matvec_noalloc).

It exists for callers that may not allocate device memory while they run,
such as code inside an external memory pool or a loop that must not take an
allocation's implicit synchronisation. It must give the same product as
gpb_forward_matvec, call after call, since every call reuses one fixed
scratch array. This file is collected last so a stop-at-first-failure run has
already run every other test.
"""
import ctypes as C

import numpy as np
import pytest

from mojogp_b200 import _lib
from mojogp_b200.kernel import RBF, make_ard_kernel
from mojogp_b200.provider import DeviceBuffer, Provider

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return float(np.linalg.norm(a - b) / np.linalg.norm(b))


def test_noalloc_matches_forward_matvec_twice(gpb_lib):
    rng = np.random.default_rng(21)
    n, d, t = 5000, 16, 16
    X = rng.standard_normal((n, d)).astype(np.float32)
    k = make_ard_kernel(RBF(ard=True), d)
    p = rng.uniform(0.5, 3.0, size=d + 1).astype(np.float32)
    prov = Provider(X, k, p, 0.01)
    for call in range(2):
        V = rng.standard_normal((t, n)).astype(np.float32)
        vd = DeviceBuffer.from_host(V)
        ref_d = DeviceBuffer((t, n))
        got_d = DeviceBuffer((t, n))
        prov.forward_matvec(ref_d, vd, t)
        _lib.call("gpb_forward_matvec_noalloc", prov.h, got_d.cptr, vd.cptr, t)
        prov.synchronize()
        ref, got = ref_d.download(), got_d.download()
        assert np.all(np.isfinite(got))
        assert _rel(got, ref) < 1e-5, f"call {call}"


def test_noalloc_rejects_oversize(gpb_lib):
    rng = np.random.default_rng(22)
    n, d = 400_000, 16
    X = rng.standard_normal((n, d)).astype(np.float32)
    k = make_ard_kernel(RBF(ard=True), d)
    prov = Provider(X, k, np.ones(d + 1, np.float32), 0.01)
    vd = DeviceBuffer((1, n))
    od = DeviceBuffer((1, n))
    st = _lib.lib().gpb_forward_matvec_noalloc(prov.h, od.cptr, vd.cptr, 1)
    assert st == _lib.ERR_INVALID
    assert "scratch" in _lib.last_error()
