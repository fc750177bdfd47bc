"""Both Gram tile kernels meet the 1e-5 matvec bar against the float64 oracle
for every Gram leaf, whichever the default picks: GPB_KV_GRAMH=0 runs the tf32
kernel (kv_tiles_gram.cuh) everywhere, GPB_KV_GRAMH=2 the fp16 kernel
(kv_tiles_gramh.cuh) everywhere (by default RBF takes the fp16 kernel and the
Matern / RQ leaves the tf32 one). The switch is read once per process, so each
mode runs in a child process."""
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
from mojogp_b200.kernel import RBF, RQ, Matern32, Matern52, make_ard_kernel
from mojogp_b200.provider import Provider
from oracle import kernels as ok
rng = np.random.default_rng(3)
want = sys.argv[2]
for ctor, d in ((RBF, 16), (Matern52, 8), (Matern32, 16), (RQ, 8)):
    n, t = 3000, 16
    X = rng.standard_normal((n, d)).astype(np.float32)
    k = make_ard_kernel(ctor(ard=True), d)
    names = k.resolve_ard(d).get_param_names()
    p = np.array([rng.uniform(1.5, 3.0) if ("length" in nm or "_ls_" in nm) else 1.2
                  for nm in names], np.float32)
    prov = Provider(X, k, p, 0.01)
    assert prov.matvec_layout(t) == want, prov.matvec_layout(t)
    V = rng.standard_normal((n, t)).astype(np.float32)
    ref = ok.forward_matvec(k.to_spec(d), p, X, V, noise=0.01)
    got = prov.matvec_host(V)
    err = float(np.linalg.norm(got - ref) / np.linalg.norm(ref))
    assert err < 1e-5, err
print("ok")
"""


@pytest.mark.parametrize("mode,layout", [("0", "gram-tensor-core-tf32"),
                                         ("2", "gram-tensor-core")])
def test_gram_kernel_modes(gpb_lib, mode, layout):
    env = dict(os.environ, GPB_KV_GRAMH=mode)
    r = subprocess.run([sys.executable, "-c", CHILD, str(ROOT), layout], env=env,
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0 and "ok" in r.stdout, r.stdout[-2000:] + r.stderr[-2000:]
