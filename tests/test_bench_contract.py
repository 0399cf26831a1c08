"""The bench's reference arm (``bench.py --impl reference``) on the host: the
reference's attention as the FP64 oracle port, timed on host threads. Its one
JSON line keeps the contract the driver reads: BASELINE's metric, the unit and
direction of this repository's own line, the same ``config`` as the headline
workload, a ``cpu_baseline`` describing the run and an ``e2e`` with no transfers.
"""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import bench  # noqa: E402


def test_reference_arm_prints_one_contract_line():
    r = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1", "--warmup", "3"], cwd=ROOT,
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = r.stdout.strip().splitlines()
    assert len(lines) == 1, r.stdout
    d = json.loads(lines[0])
    with open(os.path.join(ROOT, "BASELINE.json")) as f:
        assert d["metric"] == json.load(f)["metric"]
    assert d["impl"] == "reference"
    assert (d["unit"], d["higher_is_better"], d["n_gpus"], d["steps"]) == ("TFLOP/s", True, 1, 1)
    assert d["config"] == bench.headline_config(1)
    assert d["value"] > 0 and d["ms_per_step"] > 0
    cpu = d["cpu_baseline"]
    assert cpu["kind"] == "port" and cpu["cores"] >= 1 and cpu["value"] == d["value"] and cpu["sample"]
    e2e = d["e2e"]
    assert (e2e["value"], e2e["unit"], e2e["h2d_bytes_per_step"], e2e["d2h_bytes_per_step"]) == (d["value"], d["unit"], 0, 0)


def test_reference_arm_other_ranks_exit_without_work():
    env = dict(os.environ, RANK="1")
    r = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--gpus", "2", "--steps", "1", "--warmup", "3"],
                       cwd=ROOT, capture_output=True, text=True, timeout=120, env=env)
    assert r.returncode == 0, r.stderr[-2000:]
    assert r.stdout.strip() == ""
