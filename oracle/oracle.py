"""TEST INFRASTRUCTURE ONLY: ctypes/numpy front end of the FP64 CPU oracle.

Only tests/, ``__graft_entry__.smoke()`` and ``bench.py``'s cpu_baseline leg may
import this module, and only to check results or to time the CPU baseline.
The product (``jade_compute_b200``) never imports it.

The C functions restate the reference's CPU references (file:line citations are
in oracle.h). The expression evaluator below restates ``Expr::code`` semantics
(src/runtime/ir.rs:111-137) on the CPU in FP32 with the emitted operation order
and no fused multiply-add, which is the bit-exact target of the CUDA lowering,
and in FP64 as the reference's tolerance oracle (src/runtime/workloads.rs:171-213).
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")
REF_DIR = os.path.join(HERE, "_ref")

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_f64p = np.ctypeslib.ndpointer(np.float64, flags="C_CONTIGUOUS")
_i64p = np.ctypeslib.ndpointer(np.int64, flags="C_CONTIGUOUS")
_sz = ctypes.c_size_t


class Validation(ctypes.Structure):
    _fields_ = [("checked_elements", _sz), ("total_elements", _sz),
                ("max_abs_error", ctypes.c_double), ("max_scaled_error", ctypes.c_double),
                ("first_bad_index", ctypes.c_int64), ("max_magnitude_error", ctypes.c_double)]


class Check(ctypes.Structure):
    _fields_ = [("elements", _sz), ("max_abs_error", ctypes.c_double),
                ("max_relative_error", ctypes.c_double), ("first_bad_index", ctypes.c_int64)]


def build() -> None:
    subprocess.run(["make", "-s", "-C", HERE, "all"], check=True)


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = ctypes.CDLL(LIB_PATH)
        L.or_values.argtypes = [_f32p, _sz, ctypes.c_uint32, ctypes.c_float]
        L.or_dot.argtypes = [_sz, _sz, _sz, _f64p, _f64p, _f64p]
        L.or_gemm_reference.argtypes = [_sz, _sz, _sz, _f32p, _f32p, _f64p, ctypes.c_int]
        L.or_gemm_rows.argtypes = [_sz, _sz, _f32p, _f32p, _i64p, _sz, _f64p, ctypes.c_int]
        L.or_gemm_fp32_sequential.argtypes = [_sz, _sz, _sz, _f32p, _f32p, _f32p, ctypes.c_int]
        L.or_validation_check.argtypes = [_sz, _sz, _sz, _f32p, _f32p, _f32p, _sz, ctypes.c_int,
                                          ctypes.c_double, ctypes.POINTER(Validation)]
        L.or_compare.argtypes = [_f32p, _f64p, _sz, ctypes.c_double, ctypes.c_double,
                                 ctypes.POINTER(Check)]
        L.or_sigmoid.argtypes = [ctypes.c_double]
        L.or_sigmoid.restype = ctypes.c_double
        L.or_swiglu.argtypes = [_sz, _f32p, _f32p, _f64p]
        L.or_normalize.argtypes = [_sz, _sz, _f32p, _f32p, ctypes.c_double, _f64p, ctypes.c_int]
        L.or_softmax.argtypes = [_sz, _sz, _f32p, _f64p, ctypes.c_int]
        L.or_axpy.argtypes = [_sz, ctypes.c_float, _f32p, _f32p, _f64p]
        L.or_axpy_fp32.argtypes = [_sz, ctypes.c_float, _f32p, _f32p, _f32p]
        L.or_add_fp32.argtypes = [_sz, _f32p, _f32p, _f32p]
        L.or_attention.argtypes = [_sz, _sz, _sz, ctypes.c_int, _f32p, _f32p, _f32p, _f64p,
                                   ctypes.c_int]
        L.or_attention_rows.argtypes = [_sz, _sz, ctypes.c_int, _f32p, _f32p, _f32p, _i64p, _i64p,
                                        _sz, _f64p, ctypes.c_int]
        L.or_mlp_rows.argtypes = [_sz, _sz, _f32p, _f32p, _f32p, _f32p, _f32p, ctypes.c_double,
                                  _i64p, _sz, _f64p, ctypes.c_int]
        L.or_attention_rows_bound.argtypes = [_sz, _sz, ctypes.c_int, _f32p, _f32p, _f32p, _i64p, _i64p,
                                              _sz, _f64p, _f64p, ctypes.c_int]
        L.or_mlp_rows_ex.argtypes = [_sz, _sz, _f32p, _f32p, _f32p, _f32p, _f32p, ctypes.c_double,
                                     _i64p, _sz, ctypes.c_int, _f64p, _f64p, ctypes.c_int]
        L.or_f32_to_bf16.argtypes = [ctypes.c_float]
        L.or_f32_to_bf16.restype = ctypes.c_uint16
        L.or_bf16_to_f32.argtypes = [ctypes.c_uint16]
        L.or_bf16_to_f32.restype = ctypes.c_float
        L.or_f32_to_f16.argtypes = [ctypes.c_float]
        L.or_f32_to_f16.restype = ctypes.c_uint16
        L.or_f16_to_f32.argtypes = [ctypes.c_uint16]
        L.or_f16_to_f32.restype = ctypes.c_float
        L.or_round_bf16_array.argtypes = [_f32p, _sz]
        L.or_omp_max_threads.restype = ctypes.c_int
        _lib = L
    return _lib


def _c(x, dt=np.float32):
    return np.ascontiguousarray(x, dtype=dt)


def max_threads() -> int:
    return lib().or_omp_max_threads()


# --- inputs ---------------------------------------------------------------
def values(n: int, seed: int, scale: float = 1.0) -> np.ndarray:
    """workloads.rs:17-27 (xorshift32)."""
    out = np.empty(n, np.float32)
    lib().or_values(out, n, seed & 0xFFFFFFFF, scale)
    return out


def validation_inputs(m: int, n: int, k: int):
    """validation.rs:5-21 (seeds 0x12345678 / 0x9abcdef1)."""
    return values(m * k, 0x12345678), values(k * n, 0x9ABCDEF1)


# --- GEMM ------------------------------------------------------------------
def dot(m, n, k, a, b):
    out = np.empty(m * n, np.float64)
    lib().or_dot(m, n, k, _c(a, np.float64), _c(b, np.float64), out)
    return out


def gemm_reference(m, n, k, a, b, threads=1):
    out = np.empty(m * n, np.float64)
    lib().or_gemm_reference(m, n, k, _c(a), _c(b), out, threads)
    return out


def gemm_rows(n, k, a, b, rows, threads=1):
    rows = _c(rows, np.int64)
    out = np.empty(len(rows) * n, np.float64)
    lib().or_gemm_rows(n, k, _c(a), _c(b), rows, len(rows), out, threads)
    return out.reshape(len(rows), n)


def gemm_fp32_sequential(m, n, k, a, b, threads=1):
    out = np.empty(m * n, np.float32)
    lib().or_gemm_fp32_sequential(m, n, k, _c(a), _c(b), out, threads)
    return out


def validation_check(m, n, k, a, b, out, budget=1 << 62, fp16=False, coef=0.0):
    r = Validation()
    rc = lib().or_validation_check(m, n, k, _c(a), _c(b), _c(out), budget, int(fp16), coef,
                                   ctypes.byref(r))
    return rc, r


def compare(actual, expected, atol, rtol):
    r = Check()
    actual = _c(actual).ravel()
    expected = _c(expected, np.float64).ravel()
    if actual.size != expected.size:
        raise ValueError("oracle length mismatch")
    rc = lib().or_compare(actual, expected, actual.size, atol, rtol, ctypes.byref(r))
    return rc, r


# --- row and elementwise ops ----------------------------------------------
def sigmoid(x: float) -> float:
    return lib().or_sigmoid(x)


def swiglu(gate, up):
    gate, up = _c(gate).ravel(), _c(up).ravel()
    out = np.empty(gate.size, np.float64)
    lib().or_swiglu(gate.size, gate, up, out)
    return out


def normalize(rows, cols, x, w, eps, threads=1):
    out = np.empty(rows * cols, np.float64)
    lib().or_normalize(rows, cols, _c(x).ravel(), _c(w).ravel(), eps, out, threads)
    return out


def softmax(rows, cols, x, threads=1):
    out = np.empty(rows * cols, np.float64)
    lib().or_softmax(rows, cols, _c(x).ravel(), out, threads)
    return out


def axpy(alpha, a, b):
    a, b = _c(a).ravel(), _c(b).ravel()
    out = np.empty(a.size, np.float64)
    lib().or_axpy(a.size, alpha, a, b, out)
    return out


def axpy_fp32(alpha, a, b):
    a, b = _c(a).ravel(), _c(b).ravel()
    out = np.empty(a.size, np.float32)
    lib().or_axpy_fp32(a.size, alpha, a, b, out)
    return out


def add_fp32(a, b):
    a, b = _c(a).ravel(), _c(b).ravel()
    out = np.empty(a.size, np.float32)
    lib().or_add_fp32(a.size, a, b, out)
    return out


# --- attention and MLP -----------------------------------------------------
def attention(bh, seq, dim, causal, q, k, v, threads=1):
    out = np.empty(bh * seq * dim, np.float64)
    lib().or_attention(bh, seq, dim, int(causal), _c(q).ravel(), _c(k).ravel(), _c(v).ravel(),
                       out, threads)
    return out


def attention_rows(seq, dim, causal, q, k, v, bh_idx, row_idx, threads=1):
    bh_idx, row_idx = _c(bh_idx, np.int64), _c(row_idx, np.int64)
    out = np.empty(len(bh_idx) * dim, np.float64)
    lib().or_attention_rows(seq, dim, int(causal), _c(q).ravel(), _c(k).ravel(), _c(v).ravel(),
                            bh_idx, row_idx, len(bh_idx), out, threads)
    return out.reshape(len(bh_idx), dim)


def attention_rows_bound(seq, dim, causal, q, k, v, bh_idx, row_idx, threads=1):
    """(reference rows, magnitude sum_j p_j*|v_j|) per output element, both
    [len(bh_idx), dim]: the error of a weighted sum whose weights and output are
    rounded to 2^-t relative is bounded by ~2^-t times the magnitude."""
    bh_idx, row_idx = _c(bh_idx, np.int64), _c(row_idx, np.int64)
    out = np.empty(len(bh_idx) * dim, np.float64)
    mag = np.empty(len(bh_idx) * dim, np.float64)
    lib().or_attention_rows_bound(seq, dim, int(causal), _c(q).ravel(), _c(k).ravel(), _c(v).ravel(),
                                  bh_idx, row_idx, len(bh_idx), out, mag, threads)
    return out.reshape(len(bh_idx), dim), mag.reshape(len(bh_idx), dim)


def mlp_rows_bf16h(width, hidden, x, norm_weight, wg, wu, wd, eps, rows, threads=1):
    """The MLP chain with h rounded to BF16 where the fused block stores it, and
    the magnitude sum_p |h_p*wd_pc| + |x_c| of each output element."""
    rows = _c(rows, np.int64)
    out = np.empty(len(rows) * width, np.float64)
    mag = np.empty(len(rows) * width, np.float64)
    lib().or_mlp_rows_ex(width, hidden, _c(x).ravel(), _c(norm_weight).ravel(), _c(wg).ravel(),
                         _c(wu).ravel(), _c(wd).ravel(), eps, rows, len(rows), 1, out, mag, threads)
    return out.reshape(len(rows), width), mag.reshape(len(rows), width)


def bounded_error(got, ref, mag, out_rel, coef):
    """Checks |got - ref| <= out_rel*|ref| + coef*mag elementwise (the output's own
    rounding plus a validation.rs-style bound on the sum). Returns (ok, max of
    |got - ref| / mag, index of the first violation or -1)."""
    got = np.asarray(got, np.float64).ravel()
    ref = np.asarray(ref, np.float64).ravel()
    mag = np.asarray(mag, np.float64).ravel()
    if not (np.isfinite(got).all() and np.isfinite(ref).all()):
        return False, float("inf"), int(np.argmin(np.isfinite(got) & np.isfinite(ref)))
    err = np.abs(got - ref)
    bad = err > out_rel * np.abs(ref) + coef * mag
    scaled = float((err / np.maximum(mag, 1e-30)).max()) if err.size else 0.0
    return (not bad.any()), scaled, int(np.argmax(bad)) if bad.any() else -1


def mlp_rows(width, hidden, x, norm_weight, wg, wu, wd, eps, rows, threads=1):
    rows = _c(rows, np.int64)
    out = np.empty(len(rows) * width, np.float64)
    lib().or_mlp_rows(width, hidden, _c(x).ravel(), _c(norm_weight).ravel(), _c(wg).ravel(),
                      _c(wu).ravel(), _c(wd).ravel(), eps, rows, len(rows), out, threads)
    return out.reshape(len(rows), width)


# --- rounding --------------------------------------------------------------
def round_bf16(x):
    x = np.array(x, dtype=np.float32, copy=True).ravel()
    lib().or_round_bf16_array(x, x.size)
    return x


def f32_to_bf16_bits(x: float) -> int:
    return lib().or_f32_to_bf16(x)


def f32_to_f16_bits(x: float) -> int:
    return lib().or_f32_to_f16(x)


def f16_bits_to_f32(h: int) -> float:
    return lib().or_f16_to_f32(h)


# --- expression IR (src/runtime/ir.rs:74-137) --------------------------------
def expr_eval_f32(expr: dict, inputs) -> np.ndarray:
    """FP32 evaluation in the emitted order: each node one IEEE FP32 operation,
    no contraction (numpy float32 ufuncs round every operation). exp nodes use
    numpy's float32 exp, so they carry a tolerance rather than bit-exactness."""
    kind = expr["kind"]
    if kind == "input":
        return np.asarray(inputs[expr["binding"]], dtype=np.float32)
    if kind == "constant":
        return np.float32(expr["value"])
    if kind in ("add", "multiply", "maximum"):
        l = expr_eval_f32(expr["left"], inputs)
        r = expr_eval_f32(expr["right"], inputs)
        with np.errstate(over="ignore", invalid="ignore"):
            if kind == "add":
                return np.add(l, r, dtype=np.float32)
            if kind == "multiply":
                return np.multiply(l, r, dtype=np.float32)
            return np.fmax(l, r).astype(np.float32)
    if kind == "negate":
        return np.negative(expr_eval_f32(expr["value"], inputs)).astype(np.float32)
    if kind == "exp":
        with np.errstate(over="ignore"):
            return np.exp(expr_eval_f32(expr["value"], inputs), dtype=np.float32)
    raise ValueError(f"unknown expression kind {kind}")


def expr_eval_f64(expr: dict, inputs) -> np.ndarray:
    kind = expr["kind"]
    if kind == "input":
        return np.asarray(inputs[expr["binding"]], dtype=np.float64)
    if kind == "constant":
        return np.float64(np.float32(expr["value"]))
    if kind in ("add", "multiply", "maximum"):
        l = expr_eval_f64(expr["left"], inputs)
        r = expr_eval_f64(expr["right"], inputs)
        if kind == "add":
            return l + r
        if kind == "multiply":
            return l * r
        return np.fmax(l, r)
    if kind == "negate":
        return -expr_eval_f64(expr["value"], inputs)
    if kind == "exp":
        return np.exp(expr_eval_f64(expr["value"], inputs))
    raise ValueError(f"unknown expression kind {kind}")


def expr_has_exp(expr: dict) -> bool:
    if expr["kind"] == "exp":
        return True
    return any(expr_has_exp(expr[c]) for c in ("left", "right", "value")
               if c in expr and isinstance(expr[c], dict))


# --- the reference's conformance cases (src/runtime/workloads.rs:56-215) ------
def _relu_expr():
    return {"kind": "maximum",
            "left": {"kind": "add",
                     "left": {"kind": "multiply", "left": {"kind": "input", "binding": 0},
                              "right": {"kind": "constant", "value": 2.5}},
                     "right": {"kind": "input", "binding": 1}},
            "right": {"kind": "constant", "value": 0.0}}


def conformance_cases():
    """Returns [(name, spec, inputs, expected_f64)] exactly as workloads.rs:56-215
    builds them (same seeds, scales, shapes and FP64 expectations)."""
    cases = []
    for n in (1, 257, 1025):
        a, b = values(n, 0x1234, 2.0), values(n, 0xABCD, 1.0)
        cases.append((f"axpy_{n}", {"op": "axpy", "len": n, "alpha": -0.375}, [a, b],
                      axpy(-0.375, a, b)))
    a, b = values(257, 0x1234, 2.0), values(257, 0xABCD, 1.0)
    cases.append(("add_257", {"op": "add", "len": 257}, [a, b],
                  a.astype(np.float64) + b.astype(np.float64)))
    gate = np.array([-1000.0, -100.0, -20.0, -1.0, 0.0, 0.25, 1.0, 20.0, 100.0, 1000.0], np.float32)
    up = values(gate.size, 0xAACC, 2.0)
    cases.append(("swiglu_extreme", {"op": "swi_glu", "len": gate.size}, [gate, up],
                  swiglu(gate, up)))
    for rows, cols in ((1, 1), (3, 17), (2, 257)):
        x, w = values(rows * cols, 0x1234, 2.0), values(cols, 0xABCD, 1.0)
        eps = np.float32(1e-5)
        cases.append((f"rmsnorm_{rows}_{cols}",
                       {"op": "rms_norm", "rows": rows, "cols": cols, "epsilon": 1e-5}, [x, w],
                       normalize(rows, cols, x, w, float(eps))))
        i = np.arange(rows * cols)
        xs = np.where(i // cols == 0, np.float32(1000.0),
                      (i % cols).astype(np.float32) * np.float32(0.25) - np.float32(10000.0)
                      ).astype(np.float32)
        cases.append((f"softmax_{rows}_{cols}", {"op": "softmax", "rows": rows, "cols": cols},
                      [xs], softmax(rows, cols, xs)))
    for m, n, k in ((1, 1, 1), (31, 47, 19), (8, 33, 65)):
        for tiled in (False, True):
            a, b = values(m * k, 0x1234, 1.0), values(k * n, 0xABCD, 1.0)
            cases.append((f"gemm_{m}_{n}_{k}_tiled_{str(tiled).lower()}",
                          {"op": "gemm", "m": m, "n": n, "k": k, "tiled": tiled}, [a, b],
                          dot(m, n, k, a.astype(np.float64), b.astype(np.float64))))
    a, b = values(257, 0x1234, 1.0), values(257, 0xABCD, 1.0)
    cases.append(("custom_fused_axpy_relu",
                   {"op": "elementwise", "len": 257, "inputs": 2, "expression": _relu_expr()},
                   [a, b], np.maximum(a.astype(np.float64) * 2.5 + b.astype(np.float64), 0.0)))
    x = values(73, 0x9988, 1.0)
    cases.append(("custom_negate_exp",
                  {"op": "elementwise", "len": 73, "inputs": 1,
                   "expression": {"kind": "exp", "value": {"kind": "negate",
                                                           "value": {"kind": "input", "binding": 0}}}},
                  [x], np.exp(-x.astype(np.float64))))
    return cases
