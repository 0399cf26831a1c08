"""Pins the CPU oracle against every known-answer vector in the reference's own
unit tests, before it is trusted as the checker of the CUDA path."""
import math
import os
import subprocess

import numpy as np
import pytest

from oracle import oracle as O
from tests.conftest import HAS_REF

REF_BUILD = os.path.join(os.path.dirname(O.__file__), "_ref")


def test_gemm_kat_and_rejections():
    # src/validation.rs:102-112
    a = np.array([1, 2, -3, 4], np.float32)
    b = np.array([1, 2, 3, 4, 5, 6], np.float32)
    c = np.array([9, 12, 15, 13, 14, 15], np.float32)
    rc, r = O.validation_check(2, 3, 2, a, b, c)
    assert rc == 0 and r.checked_elements == 6
    c[5] = 0
    assert O.validation_check(2, 3, 2, a, b, c)[0] == 1
    c[5] = np.nan
    assert O.validation_check(2, 3, 2, a, b, c, budget=1)[0] == 2
    assert O.validation_check(2, 3, 2, a, b, c, budget=0)[0] == 3
    assert list(O.gemm_reference(2, 3, 2, a, b)) == [9, 12, 15, 13, 14, 15]
    assert list(O.dot(2, 3, 2, a, b)) == [9, 12, 15, 13, 14, 15]


def test_read_alias_gemm_kat():
    # src/runtime/metal.rs:820-822: a*a with a = [1,2,3,4] (2x2)
    a = np.array([1, 2, 3, 4], np.float32)
    assert list(O.gemm_reference(2, 2, 2, a, a)) == [7, 10, 15, 22]
    assert list(O.gemm_fp32_sequential(2, 2, 2, a, a)) == [7, 10, 15, 22]


def test_mixed_chain_kat():
    # src/runtime/metal.rs:893-912: ab = a*b, shifted = ab + bias, out = shifted*b
    a = np.array([1, 2, 3, 4], np.float32)
    b = np.array([2, 0, 1, 2], np.float32)
    bias = np.array([1, -1, 2, -2], np.float32)
    ab = O.gemm_fp32_sequential(2, 2, 2, a, b)
    assert list(ab) == [4, 4, 10, 8]
    shifted = O.add_fp32(ab, bias)
    assert list(shifted) == [5, 3, 12, 6]
    assert list(O.gemm_fp32_sequential(2, 2, 2, shifted, b)) == [13, 6, 30, 12]


def test_add_chain_kat():
    # src/runtime/metal.rs:971-985
    a = np.array([0, 1, -2, 3, 1], np.float32)
    b = np.array([-1, 2, 3, -4, 7], np.float32)
    mid = O.add_fp32(a, b)
    assert list(O.add_fp32(mid, b)) == [-2, 5, 4, -5, 15]


def test_attention_kat():
    # src/runtime/metal_lab.rs:471-484
    q = np.zeros(6, np.float32)
    v = np.array([1, 2, 3, 4, 8, 9], np.float32)
    assert list(O.attention(1, 3, 2, False, q, q, v)) == [4, 5, 4, 5, 4, 5]
    assert list(O.attention(1, 3, 2, True, q, q, v)) == [1, 2, 2, 3, 4, 5]
    rows = O.attention_rows(3, 2, True, q, q, v, [0, 0], [2, 1])
    assert rows.tolist() == [[4, 5], [2, 3]]


def test_compare_rejects_wrong_and_nonfinite():
    # src/runtime/workloads.rs:536-539
    assert O.compare(np.array([0.0]), np.array([1.0]), 1e-5, 1e-5)[0] == 1
    assert O.compare(np.array([np.nan]), np.array([0.0]), 1e-5, 1e-5)[0] == 2
    rc, r = O.compare(np.array([1.0, 2.0]), np.array([1.0, 2.0 + 1e-6]), 1e-5, 1e-5)
    assert rc == 0 and r.max_abs_error > 0


def test_values_stream():
    # workloads.rs:17-27 / validation.rs:5-21: first outputs computed by hand from
    # the xorshift32 recurrence.
    s = 0x1234
    want = []
    for _ in range(4):
        s ^= (s << 13) & 0xFFFFFFFF
        s ^= s >> 17
        s ^= (s << 5) & 0xFFFFFFFF
        want.append((np.float32(s >> 8) / np.float32(16777216.0) * np.float32(2.0)
                     - np.float32(1.0)) * np.float32(2.0))
    assert O.values(4, 0x1234, 2.0).tolist() == [float(np.float32(w)) for w in want]
    # seed 0 is the degenerate fixed point of xorshift32: every output is -scale.
    assert O.values(3, 0, 1.0).tolist() == [-1.0, -1.0, -1.0]


def test_sigmoid_and_swiglu_extremes():
    assert O.sigmoid(0.0) == 0.5
    assert O.sigmoid(-1000.0) == 0.0
    assert O.sigmoid(1000.0) == 1.0
    g = np.array([-1000, -1, 0, 1, 1000], np.float32)
    u = np.ones(5, np.float32)
    out = O.swiglu(g, u)
    assert out[2] == 0 and out[4] == 1000 and abs(out[3] - 1 / (1 + math.exp(-1))) < 1e-15


def test_normalize_and_softmax_small():
    x = np.array([3, 4], np.float32)
    w = np.array([1, 2], np.float32)
    out = O.normalize(1, 2, x, w, 0.0)
    inv = 1 / math.sqrt(12.5)
    assert np.allclose(out, [3 * inv, 8 * inv], rtol=0, atol=1e-15)
    sm = O.softmax(1, 3, np.array([1000, 1000, 1000], np.float32))
    assert np.allclose(sm, [1 / 3] * 3, atol=1e-15)


def test_fp16_converter_matches_reference_exhaustively_on_grid():
    # native/fp16_test.cpp:10-33 restated: every finite binary16 value round-trips.
    for raw in range(0x10000):
        e = (raw >> 10) & 31
        if e == 31:
            continue
        v = O.f16_bits_to_f32(raw)
        assert O.f32_to_f16_bits(v) == raw
    ld = math.ldexp
    assert O.f32_to_f16_bits(1 + ld(1, -11)) == 0x3C00
    assert O.f32_to_f16_bits(1 + 3 * ld(1, -11)) == 0x3C02
    assert O.f32_to_f16_bits(ld(1, -25)) == 0
    assert O.f32_to_f16_bits(65504.0) == 0x7BFF
    assert O.f32_to_f16_bits(65520.0) == 0x7C00
    assert O.f32_to_f16_bits(float("inf")) == 0x7C00
    assert O.f32_to_f16_bits(float("nan")) == 0x7E00


@pytest.mark.skipif(not os.path.exists(os.path.join(REF_BUILD, "libref_fp16.so")),
                    reason="reference FP16 converter not built (oracle/_ref)")
def test_fp16_converter_bit_exact_against_reference_build():
    import ctypes
    ref = ctypes.CDLL(os.path.join(REF_BUILD, "libref_fp16.so"))
    ref.ref_to_fp16.argtypes = [ctypes.c_float]
    ref.ref_to_fp16.restype = ctypes.c_uint16
    rng = np.random.default_rng(0)
    bits = np.concatenate([rng.integers(0, 2**32, 200000, dtype=np.uint64).astype(np.uint32),
                           np.arange(0x33000000, 0x33000000 + 4096, dtype=np.uint32),
                           np.arange(0x387FF000, 0x38801000, dtype=np.uint32),
                           np.arange(0x477FE000, 0x47801000, dtype=np.uint32)])
    vals = bits.view(np.float32)
    for v in vals:
        if np.isnan(v):
            continue
        assert O.f32_to_f16_bits(float(v)) == ref.ref_to_fp16(float(v)), hex(v.view(np.uint32))


@pytest.mark.skipif(not os.path.exists(os.path.join(REF_BUILD, "fp16_test")),
                    reason="reference fp16_test not built")
def test_reference_fp16_test_runs():
    out = subprocess.run([os.path.join(REF_BUILD, "fp16_test")], capture_output=True, text=True,
                         check=True)
    assert "63488 finite roundtrips" in out.stdout


def test_bf16_rounding():
    assert O.f32_to_bf16_bits(1.0) == 0x3F80
    # 1 + 2^-8 is a tie between 1.0 and 1+2^-7: ties to even -> 1.0
    assert O.f32_to_bf16_bits(1 + 2**-8) == 0x3F80
    assert O.f32_to_bf16_bits(1 + 3 * 2**-8) == 0x3F82
    x = O.round_bf16([1 + 2**-9, 3.0])
    assert x.tolist() == [1.0, 3.0]


def test_conformance_cases_shapes():
    cases = O.conformance_cases()
    assert len(cases) == 19
    names = [c[0] for c in cases]
    assert names[:3] == ["axpy_1", "axpy_257", "axpy_1025"]
    assert "custom_negate_exp" in names


def test_mlp_rows_matches_full_chain():
    # workloads.rs:466-479 chain, checked against an independent numpy FP64 chain.
    m, w, h = 4, 8, 16
    x = O.values(m * w, 0x1234, 1.0)
    norm = np.ones(w, np.float32)
    wg = O.values(w * h, 0x3333, 1 / math.sqrt(w))
    wu = O.values(w * h, 0x4444, 1 / math.sqrt(w))
    wd = O.values(h * w, 0x5555, 1 / math.sqrt(h))
    got = O.mlp_rows(w, h, x, norm, wg, wu, wd, 1e-5, [0, 3])
    X = x.reshape(m, w).astype(np.float64)
    nrm = X / np.sqrt((X * X).sum(1, keepdims=True) / w + 1e-5)
    g = nrm @ wg.reshape(w, h).astype(np.float64)
    u = nrm @ wu.reshape(w, h).astype(np.float64)
    act = g / (1 + np.exp(-g)) * u
    y = act @ wd.reshape(h, w).astype(np.float64) + X
    assert np.allclose(got, y[[0, 3]], rtol=1e-12, atol=1e-12)
