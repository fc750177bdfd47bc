"""tcgen05 building blocks: one 128 x 16 x 8 kind::tf32 MMA with A from
shared memory (variant 0) and from TMEM (variant 2), checked exactly against
a float64 product of the tf32-rounded operands."""
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


@pytest.mark.parametrize("variant", [0, 2])
def test_tcgen05_tf32_mma(variant):
    rng = np.random.default_rng(11 + variant)
    a = rng.standard_normal((128, 8)).astype(np.float32)
    b = rng.standard_normal((16, 8)).astype(np.float32)
    d = np.zeros((128, 16), np.float32)
    _lib.call("gpb_tc_selftest", 0, variant, C.c_void_p(a.ctypes.data), C.c_void_p(b.ctypes.data),
              C.c_void_p(d.ctypes.data))
    ref = _tf32(a).astype(np.float64) @ _tf32(b).astype(np.float64).T
    assert np.abs(d - ref).max() <= 1e-5 * np.abs(ref).max()
