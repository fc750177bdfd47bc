"""Generate golden kernel-matrix fixtures from the reference's own evaluator.

Run in a container where the reference checkout is importable:
    python tests/golden/make_golden.py /path/to/reference

It builds kernel trees with the reference API (mojogp.RBF, Matern*, RQ,
Linear, Polynomial, +, *, scale, active_dims, make_ard_kernel), evaluates the
float64 kernel matrix with KernelNode._evaluate_recursive
(mojogp/kernel.py:756-923) on seeded inputs, and stores inputs, parameters,
the tree description, parameter names, default initial parameters, the engine
parameter count and trainable mask, and K in tests/golden/kernels.npz / .json. Inputs are chosen so
no Matern exponent reaches the -20 clamp, which the reference's NumPy
evaluator does not apply but its generated GPU code does. Periodic is left
out: the NumPy evaluator divides by l^2 while the generated GPU kernel
divides by l (expressions.py:240-284); the oracle follows the GPU formula.
"""
import json
import sys
from pathlib import Path

import numpy as np


def describe(node):
    if node.kernel_type is not None:
        d = {"kernel_type": node.kernel_type.name, "ard": bool(node.ard)}
        if node.ard_dim is not None:
            d["ard_dim"] = int(node.ard_dim)
        if node.active_dims is not None:
            d["active_dims"] = [int(x) for x in node.active_dims]
        if node.initial_values:
            d["initial_values"] = {k: float(v) for k, v in node.initial_values.items()}
        return d
    d = {"operator": node.operator, "left": describe(node.left)}
    if node.right is not None:
        d["right"] = describe(node.right)
    if node.scale_factor is not None:
        d["scale_factor"] = float(node.scale_factor)
    if node.active_dims is not None:
        d["active_dims"] = [int(x) for x in node.active_dims]
    return d


def main(ref_root: str) -> None:
    sys.path.insert(0, ref_root)
    import mojogp
    from mojogp.kernel import make_ard_kernel

    d = 3
    cases = {
        "rbf_iso": mojogp.RBF(),
        "rbf_ard": make_ard_kernel(mojogp.RBF(ard=True), d),
        "matern12_iso": mojogp.Matern12(),
        "matern12_ard": make_ard_kernel(mojogp.Matern12(ard=True), d),
        "matern32_iso": mojogp.Matern32(),
        "matern32_ard": make_ard_kernel(mojogp.Matern32(ard=True), d),
        "matern52_iso": mojogp.Matern52(),
        "matern52_ard": make_ard_kernel(mojogp.Matern52(ard=True), d),
        "rq_iso": mojogp.RQ(),
        "rq_ard": make_ard_kernel(mojogp.RQ(ard=True), d),
        "linear_iso": mojogp.Linear(),
        "polynomial_iso": mojogp.Polynomial(degree=2),
        "sum_rbf_m52": mojogp.RBF() + mojogp.Matern52(),
        "product_rbf_linear": mojogp.RBF() * mojogp.Linear(),
        "scale_rbf": 2.0 * mojogp.RBF(),
        "active_dims_sum": mojogp.RBF(active_dims=[0, 1]) + mojogp.Matern32(active_dims=[2]),
    }
    rng = np.random.default_rng(1234)
    X1 = rng.uniform(0.0, 1.0, size=(24, d))
    X2 = rng.uniform(0.0, 1.0, size=(17, d))
    out = {"X1": X1, "X2": X2}
    desc = {}
    for name, k in cases.items():
        P = k.num_params()
        params = rng.uniform(0.5, 2.0, size=P)
        if k.kernel_type is not None and k.kernel_type.name == "POLYNOMIAL":
            params[0] = 2.0  # fixed integer degree
        K11, _ = k._evaluate_recursive(X1, X1, params, 0)
        K12, _ = k._evaluate_recursive(X1, X2, params, 0)
        out[f"{name}__params"] = params
        out[f"{name}__K11"] = K11
        out[f"{name}__K12"] = K12
        desc[name] = {"tree": describe(k), "param_names": k.get_param_names(),
                      "initial_params": [float(v) for v in k.get_initial_params()],
                      "engine_num_params": int(k.engine_num_params()),
                      "engine_trainable_mask": [bool(v) for v in k.engine_trainable_mask()]}
    here = Path(__file__).resolve().parent
    np.savez_compressed(here / "kernels.npz", **out)
    (here / "kernels.json").write_text(json.dumps(desc, indent=1, sort_keys=True))
    print("wrote", here / "kernels.npz")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_golden.py <path of the reference checkout>")
    main(sys.argv[1])
