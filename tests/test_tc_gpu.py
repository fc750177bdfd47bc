"""tcgen05 building blocks: one 128 x 16 x 8 kind::tf32 MMA with A from
shared memory (variant 0) and from TMEM (variant 2), checked against a
float64 product of the tf32-rounded operands; variant 3 leaves A in full
fp32 in TMEM and checks that the tensor core truncates it to tf32 (the Gram
kernel stores kernel values unrounded and relies on this)."""
import ctypes as C

import numpy as np
import pytest

from mojogp_b200 import _lib

pytestmark = pytest.mark.gpu


def _tf32(a):
    """Round-to-nearest-away tf32 (cvt.rna) of float32 values."""
    u = a.astype(np.float32).view(np.uint32).astype(np.uint64)
    u = ((u + 0x1000) & 0xFFFFE000).astype(np.uint32)
    return u.view(np.float32)


def _tf32_trunc(a):
    u = a.astype(np.float32).view(np.uint32) & np.uint32(0xFFFFE000)
    return u.view(np.float32)


@pytest.mark.parametrize("variant", [0, 2, 3])
def test_tcgen05_tf32_mma(variant):
    rng = np.random.default_rng(11 + variant)
    a = rng.standard_normal((128, 8)).astype(np.float32)
    b = rng.standard_normal((16, 8)).astype(np.float32)
    d = np.zeros((128, 16), np.float32)
    _lib.call("gpb_tc_selftest", 0, variant, C.c_void_p(a.ctypes.data), C.c_void_p(b.ctypes.data),
              C.c_void_p(d.ctypes.data))
    a_eff = _tf32_trunc(a) if variant == 3 else _tf32(a)
    ref = a_eff.astype(np.float64) @ _tf32(b).astype(np.float64).T
    assert np.abs(d - ref).max() <= 1e-5 * np.abs(ref).max()
