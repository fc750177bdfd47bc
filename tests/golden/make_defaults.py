"""Generate the golden solver-default fixtures from the reference's own Python.

Run where the reference checkout is importable:
    python tests/golden/make_defaults.py <path of the reference checkout>

It records SingleOutputGP._PRESETS (mojogp/gp.py:790-818), the LOVE rank rule
_prediction_lanczos_rank (gp.py:112-138) and the prediction solver settings
_prediction_solver_config (gp.py:141-199) for continuous (not mixed) kernels
on a grid of training settings and overrides, and the LMC initial parameters
built from lengthscales (_build_lmc_initial_params_from_lengthscales,
multi_output_gp.py:231-284), into tests/golden/defaults.json.
"""
import itertools
import json

import numpy as np
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
    # LMC initial parameters from lengthscales (multi_output_gp.py:231-284).
    from mojogp import Kernel
    from mojogp.kernel import make_ard_kernel
    from mojogp.multi_output_gp import _build_lmc_initial_params_from_lengthscales as build

    def make(spec, d, ard):
        ks = []
        for name, dims in spec:
            k = getattr(Kernel, name)(active_dims=dims) if dims else getattr(Kernel, name)()
            ks.append(make_ard_kernel(k, d) if ard else k)
        return ks

    lmc_cases = [
        ([("rbf", None), ("matern52", None)], 3, False, [0.4, 1.7]),
        ([("rbf", [0, 2]), ("matern52", [1, 3, 4])], 5, True, [0.2, 0.3, 1.1, 1.2, 1.3]),
        ([("rbf", None), ("matern32", None)], 3, True, [[0.5, 0.6, 0.7], [1.5, 1.6, 1.7]]),
        ([("rbf", None), ("rq", None), ("linear", None)], 2, False, [0.5, 0.9]),
        ([("rbf", [0, 2]), ("matern52", [1, 3, 4])], 5, True, [[1.0, 1.0], [1.0, 1.0]]),
    ]
    out["lmc_lengthscales"] = []
    for spec, d, ard, vals in lmc_cases:
        try:
            res = {"params": [float(v) for v in build(make(spec, d, ard), np.asarray(vals))]}
        except ValueError as e:
            res = {"error": str(e)}
        out["lmc_lengthscales"].append({"kernels": spec, "d": d, "ard": ard, "values": vals, **res})
    here = Path(__file__).resolve().parent
    (here / "defaults.json").write_text(json.dumps(out, indent=1, sort_keys=True))
    print("wrote", here / "defaults.json")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_defaults.py <path of the reference checkout>")
    main(sys.argv[1])
