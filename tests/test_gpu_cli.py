"""GPU runs of the `jade-runtime` CLI (src/bin/jade-runtime.rs:41-314), the
reference's conformance entry point: info, verify, metal-verify, metal-gemm,
metal-attention and mlp, each report parsed and checked (the CPU suite covers
emit and emit-suite). The metal-attention report carries the online-versus-
materialized timing ratio and the materialized path's scratch bytes that
src/runtime/metal_lab.rs:385-392 reports."""
import json
import os
import subprocess

import pytest

import jade_compute_b200 as jc

pytestmark = pytest.mark.gpu
CLI = os.path.join(os.path.dirname(jc.library_path()), "..", "bin", "jade-runtime")


def run_cli(*args, tmp_path=None, timeout=600):
    report = None
    cmd = [CLI, *args]
    if tmp_path is not None:
        report = tmp_path / "report.json"
        cmd += ["--report", str(report)]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=timeout)
    assert r.returncode == 0, (args, r.stdout[-2000:], r.stderr[-2000:])
    return json.loads(report.read_text() if report is not None else r.stdout)


def test_cli_info():
    j = run_cli("info")
    assert "B200" in json.dumps(j["runtime"])


def test_cli_verify(tmp_path):
    j = run_cli("verify", tmp_path=tmp_path)
    assert j["passed"] is True and j["checks"], j.keys()


def test_cli_metal_verify(tmp_path):
    j = run_cli("metal-verify", tmp_path=tmp_path)
    assert j["passed"] is True
    assert j["gemm_shapes"] and j["attention_shapes"] and j["fp32_precision_probes"]


def test_cli_metal_gemm(tmp_path):
    j = run_cli("metal-gemm", "--m", "512", "--n", "512", "--k", "512", "--repeats", "5", "--samples", "5", tmp_path=tmp_path)
    assert j["passed"] is True and j["shape"]["m"] == 512


@pytest.mark.parametrize("causal", [False, True], ids=["full", "causal"])
def test_cli_metal_attention_ratio_and_scratch(tmp_path, causal):
    args = ["metal-attention", "--heads", "4", "--sequence", "256", "--head-dim", "64", "--repeats", "5", "--samples", "5"]
    j = run_cli(*(args + (["--causal"] if causal else [])), tmp_path=tmp_path)
    assert j["passed"] is True
    scratch = j["logical_global_scratch_bytes"]
    assert scratch["materialized_reference"] == 2 * 4 * 256 * 256 * 4 and scratch["online_simt"] == 0
    ratio = j["ratio_materialized_to_online_gpu"]
    assert ratio > 0
    print(f"metal-attention {'causal' if causal else 'full'} 4x256x64: materialized/online GPU time {ratio:.2f}, "
          f"host {j['ratio_materialized_to_online_host']:.2f}, materialized scratch {scratch['materialized_reference']} B")


@pytest.mark.parametrize("mode", ["register", "simd", "mps"])
def test_cli_mlp(tmp_path, mode):
    args = ["mlp", "--batch", "8", "--width", "128", "--hidden", "256", "--repeats", "5", "--samples", "3"]
    if mode != "register":
        args.append(f"--{mode}-gemm")
    j = run_cli(*args, tmp_path=tmp_path)
    assert j["gemm_mode"] == mode
    assert j["initial_check"] and j["final_check"]
    assert j["ratio_separate_to_batched"] > 0
