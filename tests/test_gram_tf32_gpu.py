"""The tf32 Gram tile kernel (kv_tiles_gram.cuh), which the fp16 one replaced as
the default, stays selectable with GPB_KV_GRAMH=0 and must still meet the
1e-5 matvec bar against the float64 oracle. The switch is read once per
process, so the check runs in a child process."""
import os
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parent.parent

CHILD = r"""
import sys
import numpy as np
sys.path.insert(0, sys.argv[1])
from mojogp_b200.kernel import RBF, Matern52, make_ard_kernel
from mojogp_b200.provider import Provider
from oracle import kernels as ok
rng = np.random.default_rng(3)
for ctor, d in ((RBF, 16), (Matern52, 8)):
    n, t = 3000, 16
    X = rng.standard_normal((n, d)).astype(np.float32)
    k = make_ard_kernel(ctor(ard=True), d)
    p = np.concatenate([rng.uniform(1.5, 3.0, size=d), [1.2]]).astype(np.float32)
    prov = Provider(X, k, p, 0.01)
    assert prov.matvec_layout(t) == "gram-tensor-core-tf32", prov.matvec_layout(t)
    V = rng.standard_normal((n, t)).astype(np.float32)
    ref = ok.forward_matvec(k.to_spec(d), p, X, V, noise=0.01)
    got = prov.matvec_host(V)
    err = float(np.linalg.norm(got - ref) / np.linalg.norm(ref))
    assert err < 1e-5, err
print("ok")
"""


def test_tf32_gram_kernel_selectable(gpb_lib):
    env = dict(os.environ, GPB_KV_GRAMH="0")
    r = subprocess.run([sys.executable, "-c", CHILD, str(ROOT)], env=env, capture_output=True,
                       text=True, timeout=600)
    assert r.returncode == 0 and "ok" in r.stdout, r.stdout[-2000:] + r.stderr[-2000:]
