"""The no-allocation forward matvec (gpb_forward_matvec_noalloc).

It exists for callers that may not allocate device memory while they run,
such as code inside an external memory pool or a loop that must not take an
allocation's implicit synchronisation. It must give the same product as
gpb_forward_matvec (and the fp64 oracle), call after call, since every call
reuses one fixed scratch array, and a call after the first must not change
the device's free memory. This file is collected last so a
stop-at-first-failure run has already run every other test.
"""
import ctypes as C

import numpy as np
import pytest

from mojogp_b200 import _lib
from mojogp_b200.kernel import RBF, Matern32, Matern52, make_ard_kernel
from mojogp_b200.provider import DeviceBuffer, Provider
from oracle import kernels as ok

pytestmark = pytest.mark.gpu


def _rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / np.linalg.norm(b))


def _noalloc(prov, out, v, ncols):
    _lib.call("gpb_forward_matvec_noalloc", prov.h, out.cptr, v.cptr, ncols)


def _free_bytes():
    free, total = C.c_int64(), C.c_int64()
    _lib.call("gpb_device_mem_info", 0, C.byref(free), C.byref(total))
    return free.value


@pytest.mark.parametrize("n,d,t,kern,stale", [
    (5000, 16, 16, "rbf", False),    # Gram layout, one chunk
    (5000, 16, 16, "rbf", True),     # stale prescaled inputs: prescale + norm check in scratch
    (3000, 24, 20, "m52", False),    # DP = 32: tensor-core chunk + 4-column paired-row chunk
    (3000, 24, 24, "rbf", True),     # DP = 32: the 8-column tail chunk is the widest (80 floats)
    (2500, 8, 33, "m32", False),     # DP = 8 Gram: 16 + 16 + 1-column narrow chunk
])
def test_noalloc_matches_forward_matvec_and_oracle(gpb_lib, n, d, t, kern, stale):
    rng = np.random.default_rng(21 + n + d + t)
    X = rng.standard_normal((n, d)).astype(np.float32)
    base = {"rbf": RBF, "m52": Matern52, "m32": Matern32}[kern](ard=True)
    k = make_ard_kernel(base, d)
    lo = 0.8 if kern == "rbf" else 1.5
    names = k.resolve_ard(d).get_param_names()
    p = np.array([rng.uniform(lo, 3.0) if ("length" in nm or "_ls_" in nm) else 1.3
                  for nm in names], np.float32)
    prov = Provider(X, k, p, 0.01)
    vs = [rng.standard_normal((t, n)).astype(np.float32) for _ in range(2)]
    vds = [DeviceBuffer.from_host(V) for V in vs]
    refs = [DeviceBuffer((t, n)) for _ in range(2)]
    gots = [DeviceBuffer((t, n)) for _ in range(2)]
    if not stale:
        prov.forward_matvec(refs[0], vds[0], t)
    for call in range(2):
        if stale:
            prov.update_params(p)  # marks the prescaled inputs stale
        _noalloc(prov, gots[call], vds[call], t)
        prov.synchronize()
        got = gots[call].download()
        prov.forward_matvec(refs[call], vds[call], t)
        prov.synchronize()
        ref = refs[call].download()
        assert np.all(np.isfinite(got))
        assert _rel(got, ref) < 1e-5, f"call {call}: vs gpb_forward_matvec"
        rows = np.unique(np.concatenate([np.arange(64), rng.choice(n, 192, replace=False)]))
        orc = ok.forward_matvec(k.to_spec(d), p, X, vs[call].T, noise=0.01, rows=rows)
        assert _rel(got[:, rows].T, orc) < 1e-5, f"call {call}: vs fp64 oracle"


def test_noalloc_allocates_nothing_after_first_call(gpb_lib):
    rng = np.random.default_rng(23)
    n, d, t = 20000, 16, 16
    X = rng.standard_normal((n, d)).astype(np.float32)
    k = make_ard_kernel(RBF(ard=True), d)
    p = np.concatenate([rng.uniform(0.8, 3.0, size=d), [1.0]]).astype(np.float32)
    prov = Provider(X, k, p, 0.01)
    vd = DeviceBuffer.from_host(rng.standard_normal((t, n)).astype(np.float32))
    outs = [DeviceBuffer((t, n)) for _ in range(3)]
    _noalloc(prov, outs[0], vd, t)  # first call: loads the module holding the scratch array
    prov.synchronize()
    before = _free_bytes()
    _noalloc(prov, outs[1], vd, t)
    _noalloc(prov, outs[2], vd, t)
    prov.synchronize()
    after = _free_bytes()
    assert after == before, f"free device memory moved by {before - after} bytes"
    a, b, c = (o.download() for o in outs)
    assert _rel(b, a) < 1e-6 and _rel(c, a) < 1e-6


@pytest.mark.parametrize("n,d,ncols", [
    (400_000, 16, 1),     # far beyond the array
    (110_000, 32, 24),    # first chunk (T = 16, 64 floats/row) fits; the 8-column tail (80) does not
])
def test_noalloc_rejects_oversize(gpb_lib, n, d, ncols):
    rng = np.random.default_rng(22)
    X = rng.standard_normal((n, d)).astype(np.float32)
    k = make_ard_kernel(RBF(ard=True), d)
    prov = Provider(X, k, np.ones(d + 1, np.float32), 0.01)
    vd = DeviceBuffer((ncols, n))
    od = DeviceBuffer((ncols, n))
    st = _lib.lib().gpb_forward_matvec_noalloc(prov.h, od.cptr, vd.cptr, ncols)
    assert st == _lib.ERR_INVALID
    assert "scratch" in _lib.last_error()
