"""Generate a saved-model fixture with the reference's own SingleOutputGP.save.

Run where the reference checkout is importable:
    python tests/golden/make_saved_model.py <path of the reference checkout>

It builds a reference SingleOutputGP(RBF(ard=True)) on 96 seeded 3-D points,
sets a hand-chosen trained state (parameters, noise, mean, NLL, iteration
count, Lanczos rank) without training (the reference's engine is Mojo and does
not run here), and calls the reference's save() (mojogp/gp.py:3648-3723),
which writes tests/golden/ref_rbf_ard_config.json and
tests/golden/ref_rbf_ard_arrays.npz. tests/test_saved_model_cpu.py and
tests/test_gp_gpu.py load that artifact.
"""
import sys
from pathlib import Path

import numpy as np


def main(ref: str) -> None:
    sys.path.insert(0, ref)
    from mojogp.gp import SingleOutputGP, TrainingResult
    from mojogp.kernel import RBF, make_ard_kernel

    rng = np.random.default_rng(2024)
    n, d = 96, 3
    X = rng.uniform(-1.0, 1.0, size=(n, d)).astype(np.float32)
    y = (np.sin(2.0 * X[:, 0]) + 0.5 * X[:, 1] ** 2 - X[:, 2]
         + 0.05 * rng.standard_normal(n)).astype(np.float32)
    gp = SingleOutputGP(RBF(ard=True))
    gp.dim = d
    gp._cont_dim = d
    gp.kernel = make_ard_kernel(gp._kernel_pre_ard, d)
    gp._X_train, gp._y_train = X, y
    gp._is_trained = True
    gp._training_method = "matrix_free"
    params = np.array([0.7, 1.1, 1.6, 1.3], np.float32)  # 3 lengthscales, outputscale
    gp._training_result = TrainingResult(
        params=params, noise=0.004, mean=0.12, nll=-0.85, iterations=50, converged=False,
        lanczos_root=None, lanczos_rank=30)
    out = Path(__file__).resolve().parent / "ref_rbf_ard"
    gp.save(str(out))
    print("wrote", out.name + "_config.json", out.name + "_arrays.npz")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "/root/reference")
