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
