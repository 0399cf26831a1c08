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
    assert "jade_elementwise" in src and "float4" in src
    assert "__fmul_rn" in src and "__fadd_rn" in src and "fmaf" not in src
    rejects({"op": "add", "len": 4}, lambda s: jc.emit(s, "cuda"))


def test_create_without_gpu_fails_cleanly():
    if jc.device_count() > 0:
        pytest.skip("GPU present")
    with pytest.raises(JadeError) as e:
        jc.Runtime(0)
    assert e.value.code in (1, 2)
