"""bench.py's reference arm (the reference's CPU route on the host cores) keeps
the driver's JSON-line contract: one line from rank 0, nothing from other
ranks, the metric / unit / direction of the GPU arm, a cpu_baseline object and
an e2e object with zero copy bytes. Small n so the run takes seconds."""
import json
import os
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
CMD = [sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--rows", "3000",
       "--steps", "3", "--warmup", "3"]


def _run(env_extra):
    env = dict(os.environ, **env_extra)
    return subprocess.run(CMD, cwd=ROOT, env=env, capture_output=True, text=True, timeout=300)


def test_reference_arm_prints_one_contract_line():
    r = _run({"RANK": "0", "WORLD_SIZE": "1"})
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1
    line = json.loads(lines[0])
    assert line["impl"] == "reference"
    assert line["metric"].startswith("kernel-matvec TFLOP/s") and line["unit"] == "TFLOP/s"
    assert line["higher_is_better"] is True and line["steps"] == 3 and line["warmup"] == 3
    assert line["value"] > 0 and line["cpu_baseline"]["value"] == line["value"]
    # "reference" when the reference package is installed under baseline/_ref
    # (its own KernelNode.evaluate is timed), else "port" (the restatement).
    ref_installed = (ROOT / "baseline" / "_ref" / "mojogp" / "kernel.py").exists()
    assert line["cpu_baseline"]["kind"] == ("reference" if ref_installed else "port")
    assert line["cpu_baseline"]["cores"] >= 1
    assert line["e2e"] == {"value": line["value"], "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}
    assert line["config"]["n"] == 3000 and line["config"]["t"] == 16


def test_reference_arm_other_ranks_are_silent():
    r = _run({"RANK": "1", "WORLD_SIZE": "2"})
    assert r.returncode == 0 and r.stdout.strip() == ""
