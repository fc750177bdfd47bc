"""Saved-model artifacts in the reference's layout (mojogp/gp.py:3648-3910),
without a GPU: the fixture written by the reference's own save()
(tests/golden/make_saved_model.py) passes the reference's checks, the checks
reject other wrappers and schema versions with the reference's messages, and
the config written here carries every key the reference's load() reads."""
import json
import shutil
from pathlib import Path

import numpy as np
import pytest

from mojogp_b200.gp import SingleOutputGP, TrainingResult
from mojogp_b200.kernel import KernelNode, RBF

GOLDEN = Path(__file__).resolve().parent / "golden"


def test_reference_fixture_reads():
    cfg, arr = SingleOutputGP.read_artifact(str(GOLDEN / "ref_rbf_ard"))
    assert cfg["wrapper"] == "SingleOutputGP" and cfg["schema_version"] == 1
    assert arr["X_train"].shape == (96, 3) and arr["params"].shape == (4,)
    k = KernelNode.from_dict(cfg["kernel_tree"])
    assert k.has_ard() and k.kernel_type.name == "RBF"
    assert k.resolve_ard(3).num_params() == 4
    # the ".json" / ".npz" suffix is dropped as in the reference
    cfg2, _ = SingleOutputGP.read_artifact(str(GOLDEN / "ref_rbf_ard.json"))
    assert cfg2 == cfg


@pytest.mark.parametrize("edit,msg", [
    ({"wrapper": "MultiOutputGP"}, "Saved model is not a SingleOutputGP artifact"),
    ({"schema_version": 2}, "Unsupported SingleOutputGP schema_version=2"),
])
def test_reference_checks(tmp_path, edit, msg):
    cfg = json.loads((GOLDEN / "ref_rbf_ard_config.json").read_text())
    cfg.update(edit)
    (tmp_path / "m_config.json").write_text(json.dumps(cfg))
    shutil.copy(GOLDEN / "ref_rbf_ard_arrays.npz", tmp_path / "m_arrays.npz")
    with pytest.raises(ValueError, match=msg):
        SingleOutputGP.read_artifact(str(tmp_path / "m"))


def test_missing_kernel_tree(tmp_path):
    cfg = json.loads((GOLDEN / "ref_rbf_ard_config.json").read_text())
    del cfg["kernel_tree"]
    (tmp_path / "m_config.json").write_text(json.dumps(cfg))
    shutil.copy(GOLDEN / "ref_rbf_ard_arrays.npz", tmp_path / "m_arrays.npz")
    with pytest.raises(ValueError, match="missing required kernel_tree"):
        SingleOutputGP.read_artifact(str(tmp_path / "m"))


def test_written_config_has_reference_keys():
    ref = json.loads((GOLDEN / "ref_rbf_ard_config.json").read_text())
    gp = SingleOutputGP(RBF(ard=True))
    gp.dim = 3
    gp._training_method = "matrix_free"
    gp._training_result = TrainingResult(params=np.ones(4, np.float32), noise=0.004, mean=0.12,
                                         nll=-0.85, iterations=50, converged=False,
                                         lanczos_root=None, lanczos_rank=30)
    ours = gp._artifact_config()
    # kernel_mojo_type names the reference's compiled Mojo kernel and is not read by its load().
    assert set(ref) - set(ours) == {"kernel_mojo_type"}
    for key in ("wrapper", "schema_version", "dim", "ard", "cat_dims", "cat_kernel",
                "noise_mode", "result_type", "noise", "mean", "nll", "iterations", "converged",
                "lanczos_rank", "kernel_tree", "is_mixed"):
        assert ours[key] == ref[key], key
