"""Pin the oracle's kernel formulas to the reference's fp64 evaluator.

Golden fixtures come from mojogp/kernel.py:_evaluate_recursive, produced by
tests/golden/make_golden.py. The trees are rebuilt with this package's kernel
objects and encoded to the device program, so the test also pins the
parameter layout and the spec encoding.
"""
import json
from pathlib import Path

import numpy as np
import pytest

from mojogp_b200.kernel import KernelNode
from oracle import kernels as ok

GOLDEN = Path(__file__).resolve().parent / "golden"
DESC = json.loads((GOLDEN / "kernels.json").read_text())
DATA = np.load(GOLDEN / "kernels.npz")


@pytest.mark.parametrize("name", sorted(DESC))
def test_oracle_matches_reference_evaluator(name):
    tree = KernelNode.from_dict(DESC[name]["tree"])
    assert tree.get_param_names() == DESC[name]["param_names"]
    spec = tree.to_spec(DATA["X1"].shape[1])
    params = DATA[f"{name}__params"]
    K11 = ok.kernel_matrix(spec, params, DATA["X1"])
    K12 = ok.kernel_matrix(spec, params, DATA["X1"], DATA["X2"])
    # The reference forms squared distances by the expansion |x|^2+|y|^2-2x.y,
    # so coincident points get r ~ 1e-8 instead of 0 (visible through sqrt in
    # the Matern-1/2 kernel): 1e-7 relative covers that, everything else
    # agrees to ~1e-15.
    np.testing.assert_allclose(K11, DATA[f"{name}__K11"], rtol=1e-7, atol=1e-10)
    np.testing.assert_allclose(K12, DATA[f"{name}__K12"], rtol=1e-7, atol=1e-10)


@pytest.mark.parametrize("name", ["rbf_ard", "matern52_iso", "rq_ard", "sum_rbf_m52",
                                  "product_rbf_linear", "scale_rbf", "active_dims_sum",
                                  "polynomial_iso", "matern12_ard", "linear_iso"])
def test_oracle_gradients_match_finite_differences(name):
    tree = KernelNode.from_dict(DESC[name]["tree"])
    X = DATA["X1"][:10]
    spec = tree.to_spec(X.shape[1])
    params = DATA[f"{name}__params"].astype(np.float64)
    mask = tree.engine_trainable_mask()
    _, G = ok.kernel_matrix(spec, params, X, want_grad=True)
    for p in range(len(params)):
        if not mask[p]:
            continue
        h = 1e-6 * max(1.0, abs(params[p]))
        pp, pm = params.copy(), params.copy()
        pp[p] += h
        pm[p] -= h
        fd = (ok.kernel_matrix(spec, pp, X) - ok.kernel_matrix(spec, pm, X)) / (2 * h)
        np.testing.assert_allclose(G[p], fd, rtol=1e-5, atol=1e-7)


@pytest.mark.parametrize("name", sorted(DESC))
def test_default_parameters_and_trainable_mask_match_reference(name):
    """Default initial parameters (KernelNode.get_initial_params) and which
    parameters Adam moves (engine_trainable_mask, mojogp/kernel.py:482-492).
    The reference's polynomial engine layout carries one hidden leading slot
    (fixed variance), so only its public tail is compared."""
    tree = KernelNode.from_dict(DESC[name]["tree"])
    np.testing.assert_array_equal(tree.get_initial_params(), DESC[name]["initial_params"])
    ref_mask = np.array(DESC[name]["engine_trainable_mask"])
    ours = tree.engine_trainable_mask()
    assert list(ours) == list(ref_mask[len(ref_mask) - len(ours):])
