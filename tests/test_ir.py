"""CPU tests of the checked IR and emitters behind the C ABI: the reference's own
IR unit tests (src/runtime/ir.rs:578-703) restated, and byte-exact CoreX emission
against the reference's committed emit-suite output (tests/golden/emitter.json)."""
import hashlib
import json
import os

import pytest

import jade_compute_b200 as jc
from jade_compute_b200.runtime import JadeError
from oracle import oracle as O
from tests.conftest import HAS_REF, REF_ROOT

GOLDEN = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "emitter.json")))
UMAX = 2**32 - 1


def rejects(spec, fn=jc.spec_validate):
    with pytest.raises(JadeError) as e:
        fn(spec)
    assert e.value.code == 1
    return e.value.message


def test_library_exports_every_declared_symbol():
    import re
    import ctypes
    header = open(jc.runtime.INCLUDE).read()
    names = re.findall(r"^JR_API [a-z0-9_ *]+?\b(jr\w+)\(", header, re.M)
    assert len(names) >= 28
    L = ctypes.CDLL(jc.library_path())
    for n in names:
        assert hasattr(L, n), n
    assert jc.lib().jr_version() == 1 and jc.lib().jr2_version() == 2


def test_metal_specific_ops_fail_closed_on_corex_and_validate_aliases():
    # ir.rs:581-625
    specs = [{"op": "gemm_simd", "m": 33, "n": 17, "k": 65},
             {"op": "attention_online", "heads": 2, "seq": 33, "dim": 17, "causal": True},
             {"op": "attention_scores", "heads": 2, "seq": 33, "dim": 17, "causal": True},
             {"op": "attention_apply", "heads": 2, "seq": 33, "dim": 17}]
    for spec in specs:
        msg = rejects(spec, lambda s: jc.emit(s, "corex"))
        assert "Metal-only operation" in msg
        assert json.loads(jc.canonical(spec)) == spec  # serde round trip is stable
        bindings = jc.spec_bindings(spec)
        lengths = [b["elements"] for b in bindings]
        ids = list(range(len(bindings)))
        jc.spec_validate_bindings(spec, lengths, ids)
        ids[-1] = 0
        rejects(spec, lambda s: jc.spec_validate_bindings(s, lengths, ids))


@pytest.mark.parametrize("h,s,d", [(0, 1, 1), (33, 1, 1), (1, 0, 1), (1, 2049, 1), (1, 1, 0), (1, 1, 129),
                                   (UMAX, UMAX, UMAX)])
def test_attention_bounds(h, s, d):
    # ir.rs:626-643
    rejects({"op": "attention_online", "heads": h, "seq": s, "dim": d, "causal": False})


def test_gemm_simd_overflow_rejected():
    # ir.rs:644-650
    rejects({"op": "gemm_simd", "m": UMAX, "n": UMAX, "k": UMAX})


def test_expression_frontend_rejects_unbound_and_deep():
    # ir.rs:652-674
    msg = rejects({"op": "elementwise", "len": 7, "inputs": 1, "expression": {"kind": "input", "binding": 1}})
    assert "binding out of range" in msg
    rejects({"op": "elementwise", "len": 7, "inputs": 1, "expression": {"kind": "input", "binding": 1}},
            lambda s: jc.emit(s, "corex"))
    deep = {"kind": "input", "binding": 0}
    for _ in range(34):
        deep = {"kind": "negate", "value": deep}
    assert "complexity limit" in rejects({"op": "elementwise", "len": 7, "inputs": 1, "expression": deep})
    ok = {"kind": "input", "binding": 0}
    for _ in range(32):
        ok = {"kind": "negate", "value": ok}
    jc.spec_validate({"op": "elementwise", "len": 7, "inputs": 1, "expression": ok})


def test_invalid_semantics_and_aliases():
    # ir.rs:675-702
    assert "epsilon" in rejects({"op": "rms_norm", "rows": 1, "cols": 17, "epsilon": 0.0})
    assert "INT_MAX" in rejects({"op": "gemm", "m": UMAX, "n": 2, "k": 1, "tiled": True})
    spec = {"op": "add", "len": 17}
    rejects(spec, lambda s: jc.spec_validate_bindings(s, [17, 17, 17], [1, 2, 1]))
    rejects(spec, lambda s: jc.spec_validate_bindings(s, [17, 16, 17], [1, 2, 3]))
    jc.spec_validate_bindings(spec, [17, 17, 17], [1, 1, 3])  # read/read aliasing is allowed


def test_nonfinite_alpha_rejected():
    # JSON has no NaN literal; the reference rejects a non-finite alpha (ir.rs:684-689).
    assert "alpha" in rejects('{"op":"axpy","len":1,"alpha":1e39}')


def test_dimension_messages():
    assert "INT_MAX" in rejects({"op": "add", "len": 0})
    assert "31-bit" in rejects({"op": "gemm", "m": 65536, "n": 65536, "k": 1, "tiled": True})
    assert "input count" in rejects({"op": "elementwise", "len": 4, "inputs": 9,
                                     "expression": {"kind": "input", "binding": 0}})
    assert "missing field" in rejects({"op": "gemm", "m": 1, "n": 1, "k": 1})
    assert "unknown variant" in rejects({"op": "conv", "len": 1})


def test_extension_fields_validate():
    jc.spec_validate({"op": "gemm", "m": 256, "n": 256, "k": 64, "tiled": True, "dtype": "bf16"})
    jc.spec_validate({"op": "attention_online", "heads": 16, "seq": 16384, "dim": 128, "causal": True,
                      "dtype": "bf16", "batch": 4})
    rejects({"op": "attention_online", "heads": 16, "seq": 4096, "dim": 128, "causal": True})  # fp32 keeps ref limits
    rejects({"op": "attention_online", "heads": 1, "seq": 64, "dim": 96, "causal": True, "dtype": "bf16"})
    rejects({"op": "gemm", "m": 8, "n": 8, "k": 8, "tiled": True, "epilogue": "swiglu", "dtype": "bf16"})
    b = jc.spec_bindings({"op": "gemm", "m": 8, "n": 128, "k": 16, "tiled": True, "dtype": "bf16",
                          "b_layout": "nk", "epilogue": "swiglu", "row_scale": True, "out_dtype": "bf16"})
    assert [x["name"] for x in b] == ["a", "b", "row_scale", "out"]
    assert b[1]["elements"] == 2 * 128 * 16 and b[3]["dtype"] == "bf16"
    # extension specs have no reference launch geometry and no CoreX lowering
    rejects({"op": "gemm", "m": 8, "n": 8, "k": 8, "tiled": True, "dtype": "bf16"}, jc.spec_launch)
    rejects({"op": "gemm", "m": 8, "n": 8, "k": 8, "tiled": True, "dtype": "bf16"}, lambda s: jc.emit(s, "corex"))


@pytest.mark.parametrize("case", O.conformance_cases(), ids=lambda c: c[0])
def test_corex_emitter_byte_exact(case):
    name, spec, _, _ = case
    g = {c["case"]: c for c in GOLDEN["cases"]}[name]
    text = jc.emit(spec, "corex") + "\n"  # emit-suite writes content + "\n" (jade-runtime.rs:135-141)
    assert hashlib.sha256(text.encode()).hexdigest() == g["cu_sha256"], text
    if HAS_REF:  # direct diff for a readable failure where the reference tree exists
        with open(os.path.join(REF_ROOT, "reports", "generated-native", name + ".cu")) as f:
            assert f.read() == text
    metal = jc.emit(spec, "metal") + "\n"
    assert hashlib.sha256(metal.encode()).hexdigest() == g["metal_sha256"], metal
    assert jc.spec_launch(spec) == g["launch"]
    b = [{k: x[k] for k in ("elements", "name", "write")} for x in jc.spec_bindings(spec)]
    assert b == g["bindings"]
    pretty = jc.canonical(spec) + "\n"
    assert hashlib.sha256(pretty.encode()).hexdigest() == g["spec_json_sha256"], pretty


def test_cuda_lowering_is_vectorised_and_contraction_free():
    spec = O.conformance_cases()[-2][1]
    src = jc.emit(spec, "cuda")
    assert "jade_elementwise" in src and "float4" in src and "jade_generated_launch" in src
    assert "__fmul_rn" in src and "__fadd_rn" in src and "fmaf" not in src
    # the Metal-only operations and backend extensions have no cuda lowering
    rejects({"op": "attention_online", "heads": 2, "seq": 33, "dim": 17, "causal": True}, lambda s: jc.emit(s, "cuda"))
    rejects({"op": "gemm", "m": 8, "n": 8, "k": 8, "tiled": True, "dtype": "bf16"}, lambda s: jc.emit(s, "cuda"))


CLI = os.path.join(os.path.dirname(jc.library_path()), "..", "bin", "jade-runtime")


def test_cli_emit_suite_matches_the_reference_output(tmp_path):
    # jade-runtime emit-suite (src/bin/jade-runtime.rs:218-244): every case's .json,
    # .metal and CoreX .cu byte-exact to the reference's committed output and the
    # manifest's sha256, plus this backend's sm_100a module of every case
    import subprocess
    r = subprocess.run([CLI, "emit-suite", "--directory", str(tmp_path)], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0, r.stderr
    digest = lambda p: hashlib.sha256(open(p, "rb").read()).hexdigest()
    assert digest(tmp_path / "manifest.json") == GOLDEN["manifest_sha256"]
    for g in GOLDEN["cases"]:
        name = g["case"]
        assert digest(tmp_path / f"{name}.cu") == g["cu_sha256"], name
        assert digest(tmp_path / f"{name}.metal") == g["metal_sha256"], name
        assert digest(tmp_path / f"{name}.json") == g["spec_json_sha256"], name
        text = (tmp_path / f"{name}.sm100a.cu").read_text()
        assert "jade_generated_launch" in text and "sm_100a" in text, name
    assert len(list(tmp_path.glob("*.sm100a.cu"))) == len(GOLDEN["cases"])


def test_cuda_emit_target_compiles_for_sm100a(tmp_path):
    # every case's emitted sm_100a module builds with nvcc (cross-compiled here;
    # the GPU tests run them through jr_execute)
    import concurrent.futures
    import shutil
    import subprocess
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(nvcc):
        pytest.skip("nvcc not available")

    def build(case):
        name, spec = case[0], case[1]
        src = tmp_path / f"{name}.cu"
        src.write_text(jc.emit(spec, "cuda"))
        r = subprocess.run([nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-shared", "-Xcompiler", "-fPIC",
                            "-o", str(tmp_path / f"{name}.so"), str(src)], capture_output=True, text=True, timeout=300)
        return name, r.returncode, r.stderr[-2000:]

    with concurrent.futures.ThreadPoolExecutor(8) as ex:
        for name, rc, err in ex.map(build, O.conformance_cases()):
            assert rc == 0, (name, err)


def test_create_without_gpu_fails_cleanly():
    if jc.device_count() > 0:
        pytest.skip("GPU present")
    with pytest.raises(JadeError) as e:
        jc.Runtime(0)
    assert e.value.code in (1, 2)


def test_wait_probe_spec():
    spec = {"op": "wait_probe", "limit_ns": 1000000}
    jc.spec_validate(spec)
    assert [b["name"] for b in jc.spec_bindings(spec)] == ["elapsed_ns"]
    rejects({"op": "wait_probe", "limit_ns": 10})
    rejects({"op": "wait_probe", "limit_ns": 10**11})
    rejects(spec, lambda s: jc.emit(s, "corex"))
