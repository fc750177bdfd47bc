"""Solver defaults against the reference's own Python (golden fixture from
tests/golden/make_defaults.py): the fit presets, the LOVE rank rule and the
prediction solver settings a user gets without overrides."""
import json
from pathlib import Path

import pytest

from mojogp_b200.gp import SingleOutputGP, _prediction_lanczos_rank, _prediction_solver_config

GOLD = json.loads((Path(__file__).resolve().parent / "golden" / "defaults.json").read_text())


def test_presets_match_reference():
    assert SingleOutputGP._PRESETS == GOLD["presets"]


@pytest.mark.parametrize("case", GOLD["lanczos_rank"],
                         ids=lambda c: f"hint{c['rank_hint']}-ard{c['is_ard']}")
def test_love_rank_rule_matches_reference(case):
    assert _prediction_lanczos_rank(case["rank_hint"], case["is_ard"]) == case["rank"]


def test_prediction_solver_config_matches_reference():
    bad = []
    for c in GOLD["solver_config"]:
        got = _prediction_solver_config(c["train_info"], c["rank_hint"], is_ard=c["is_ard"],
                                        **c["overrides"])
        if got != c["config"]:
            bad.append((c, got))
    assert not bad, bad[:3]


def _lmc_kernels(spec, d, ard):
    from mojogp_b200.kernel import Kernel, make_ard_kernel
    ks = []
    for name, dims in spec:
        k = getattr(Kernel, name)(active_dims=dims) if dims else getattr(Kernel, name)()
        ks.append(make_ard_kernel(k, d) if ard else k.resolve_ard(d))
    return ks


@pytest.mark.parametrize("case", GOLD["lmc_lengthscales"], ids=lambda c: str(c["values"]))
def test_lmc_initial_params_from_lengthscales_match_reference(case):
    import numpy as np

    from mojogp_b200.multi_output_gp import build_lmc_initial_params_from_lengthscales
    ks = _lmc_kernels(case["kernels"], case["d"], case["ard"])
    if "error" in case:
        with pytest.raises(ValueError) as e:
            build_lmc_initial_params_from_lengthscales(ks, np.asarray(case["values"]))
        assert str(e.value) == case["error"]
    else:
        got = build_lmc_initial_params_from_lengthscales(ks, np.asarray(case["values"]))
        np.testing.assert_array_equal(got, np.asarray(case["params"], np.float32))


def test_lmc_fit_rejects_ambiguous_and_misshaped_initial_parameters():
    """Checked before any device work (multi_output_gp.py:231-284 and the
    reference's public-contract tests)."""
    import numpy as np

    from mojogp_b200.kernel import Kernel
    from mojogp_b200.multi_output_gp import MultiOutputLMCGP
    rng = np.random.default_rng(123)
    X = rng.standard_normal((8, 3)).astype(np.float32)
    Y = rng.standard_normal((8, 2)).astype(np.float32)
    gp = MultiOutputLMCGP(kernels=[Kernel.rbf()])
    with pytest.raises(ValueError, match="not both"):
        gp.fit(X, Y, initial_params=np.ones(2), initial_lengthscales=np.ones(1))
    gp = MultiOutputLMCGP(kernels=[Kernel.rbf(), Kernel.matern52()], ard=True)
    with pytest.raises(ValueError, match="initial_lengthscales"):
        gp.fit(X, Y, initial_lengthscales=np.ones((2, 2), np.float32))
    with pytest.raises(ValueError, match="initial_params has 3 values"):
        gp.fit(X, Y, initial_params=np.ones(3, np.float32))
