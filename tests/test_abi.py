"""C-ABI boundary checks that need no GPU: the library loads, exports every
symbol include/gpb200.h declares, and rejects malformed inputs on the host
side before any device work."""
import ctypes as C
from pathlib import Path

import numpy as np
import pytest

from mojogp_b200 import _lib
from mojogp_b200.kernel import RBF, Matern52, KernelNode

HEADER = Path(__file__).resolve().parent.parent / "include" / "gpb200.h"


def test_library_exports_every_declared_symbol(gpb_lib):
    declared = _lib.declared_symbols(HEADER)
    assert len(declared) >= 20
    missing = [s for s in declared if not hasattr(gpb_lib, s)]
    assert not missing, missing


def test_ctypes_signatures_cover_header(gpb_lib):
    declared = set(_lib.declared_symbols(HEADER))
    assert declared == set(_lib.SIGNATURES), declared ^ set(_lib.SIGNATURES)


def test_version_string(gpb_lib):
    assert b"gpb200" in gpb_lib.gpb_version()


def _create(spec, X, params, noise=0.1):
    h = C.c_void_p()
    st = _lib.lib().gpb_provider_create(
        C.c_void_p(X.ctypes.data), X.shape[0], X.shape[1], C.c_void_p(spec.ctypes.data),
        len(spec), C.c_void_p(params.ctypes.data), len(params), noise, None, 0, C.byref(h))
    return st, h


def test_malformed_spec_rejected_on_host(gpb_lib):
    X = np.zeros((4, 2), np.float32)
    params = np.ones(2, np.float32)
    bad = np.array([1, 2, 1, 1, 99, 0, 0, 2, 0, 1], np.int32)  # unknown kernel type
    st, h = _create(bad, X, params)
    assert st == _lib.ERR_INVALID
    assert "unknown kernel type" in _lib.last_error()


def test_param_count_mismatch_rejected(gpb_lib):
    X = np.zeros((4, 2), np.float32)
    spec = RBF().to_spec(2)
    st, _ = _create(spec, X, np.ones(3, np.float32))
    assert st == _lib.ERR_INVALID
    assert "expects" in _lib.last_error()


def test_active_dim_out_of_range_rejected(gpb_lib):
    X = np.zeros((4, 2), np.float32)
    spec = np.array([1, 2, 1, 1, 0, 0, 0, 1, 5], np.int32)
    st, _ = _create(spec, X, np.ones(2, np.float32))
    assert st == _lib.ERR_INVALID


def test_spec_encoding_layout():
    k = RBF(active_dims=[0, 2]) + 2.0 * Matern52(ard=True)
    spec = k.to_spec(3)
    # version, P, nodes
    assert spec[0] == 1 and spec[1] == k.resolve_ard(3).num_params() == 2 + 4 + 1
    assert spec[2] == 4  # leaf, leaf, scale, sum
    rt = KernelNode.from_dict(k.to_dict())
    assert np.array_equal(rt.to_spec(3), spec)


def test_host_register_rejects_bad_buffers(gpb_lib):
    assert _lib.lib().gpb_host_register(None, 16) == _lib.ERR_INVALID
    a = np.zeros(4, np.float32)
    assert _lib.lib().gpb_host_register(C.c_void_p(a.ctypes.data), 0) == _lib.ERR_INVALID
    assert _lib.lib().gpb_host_unregister(None) == _lib.ERR_INVALID
