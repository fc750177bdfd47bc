"""Generate the golden solver-default fixtures from the reference's own Python.

Run where the reference checkout is importable:
    python tests/golden/make_defaults.py <path of the reference checkout>

It records SingleOutputGP._PRESETS (mojogp/gp.py:790-818), the LOVE rank rule
_prediction_lanczos_rank (gp.py:112-138) and the prediction solver settings
_prediction_solver_config (gp.py:141-199) for continuous (not mixed) kernels
on a grid of training settings and overrides, into tests/golden/defaults.json.
"""
import itertools
import json
import sys
from pathlib import Path


def main(ref: str) -> None:
    sys.path.insert(0, ref)
    from mojogp import gp as g

    out = {"presets": g.SingleOutputGP._PRESETS, "lanczos_rank": [], "solver_config": []}
    for hint, ard in itertools.product([None, 0, 30, 150, 250, 400], [False, True]):
        out["lanczos_rank"].append({"rank_hint": hint, "is_ard": ard,
                                    "rank": g._prediction_lanczos_rank(hint, "matrix_free",
                                                                       False, ard)})
    train_infos = [None, {}, {"max_cg_iterations": 100, "cg_tolerance": 1e-2, "precond_rank": 0},
                   {"max_cg_iterations": 500, "cg_tolerance": 1e-4, "precond_rank": 64},
                   {"max_cg_iter": 40, "cg_tol": 0.5}]
    overrides = [{}, {"max_cg_iterations": 77}, {"cg_tolerance": 0.2}, {"precond_rank": 5},
                 {"max_root_decomposition_size": 33}]
    for ti, ov, hint, ard in itertools.product(train_infos, overrides, [None, 30], [False, True]):
        cfg = g._prediction_solver_config("love", ti, hint, "matrix_free", is_mixed=False,
                                          is_ard=ard, **ov)
        out["solver_config"].append({"train_info": ti, "overrides": ov, "rank_hint": hint,
                                     "is_ard": ard, "config": cfg})
    here = Path(__file__).resolve().parent
    (here / "defaults.json").write_text(json.dumps(out, indent=1, sort_keys=True))
    print("wrote", here / "defaults.json")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_defaults.py <path of the reference checkout>")
    main(sys.argv[1])
