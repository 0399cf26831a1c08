"""GPU parity of the SIMT/NVRTC kernels and the ordered-batch runtime.

Restates the reference's conformance suite (src/runtime/workloads.rs:245-320),
its batch ordering/ownership tests (src/runtime/metal.rs:776-991) and the
metal-verify shape lists (src/runtime/metal_lab.rs:398-466) against the CUDA
backend, checked with the FP64 CPU oracle. Integer/indexing and FP32 paths that
the reference computes with a fixed operation order are checked bit for bit.
"""
import ctypes
import glob
import os

import numpy as np
import pytest

import jade_compute_b200 as jc
from jade_compute_b200.runtime import JadeError, JR_EINVAL
from oracle import oracle as O

pytestmark = pytest.mark.gpu
REF_BUILD = os.path.join(os.path.dirname(O.__file__), "_ref")


@pytest.fixture(scope="module")
def rt():
    r = jc.Runtime(0)
    yield r
    r.close()


def resident(rt, data, dtype="fp32"):
    b = rt.alloc(len(data), dtype)
    rt.upload(b, data)
    return b


def run(rt, spec, inputs, repeats=2, graph=False):
    k = rt.compile(spec)
    bufs = [resident(rt, x) for x in inputs]
    out_len = jc.spec_bindings(spec)[-1]["elements"]
    out = rt.alloc(out_len)
    t = rt.execute([(k, bufs + [out])], repeats=repeats, graph=graph)
    return rt.download(out), t, k


@pytest.mark.parametrize("case", O.conformance_cases(), ids=lambda c: c[0])
def test_conformance_case(rt, case):
    # workloads.rs:245-269: every case against its FP64 expectation at 3e-5/3e-5
    name, spec, inputs, expected = case
    got, timing, k = run(rt, spec, inputs)
    rc, r = O.compare(got, expected, 3e-5, 3e-5)
    assert rc == 0, (name, r.first_bad_index, r.max_abs_error)
    assert timing.dispatches == 2 and timing.repeats == 2
    # operation-order-exact FP32 targets
    op = spec["op"]
    if op == "axpy":
        assert np.array_equal(got, O.axpy_fp32(spec["alpha"], *inputs))
    elif op == "add":
        assert np.array_equal(got, O.add_fp32(*inputs))
    elif op == "gemm":
        assert np.array_equal(got, O.gemm_fp32_sequential(spec["m"], spec["n"], spec["k"], *inputs))
    elif op == "elementwise" and not O.expr_has_exp(spec["expression"]):
        assert np.array_equal(got, O.expr_eval_f32(spec["expression"], inputs))


def test_rejections_before_any_work(rt):
    # workloads.rs:270-316: the five rejected calls
    spec = {"op": "add", "len": 17}
    k = rt.compile(spec)
    a, b, wrong = rt.alloc(17), rt.alloc(17), rt.alloc(16)
    with pytest.raises(JadeError):
        rt.upload(a, np.zeros(16, np.float32))
    with pytest.raises(JadeError):
        rt.execute([(k, [a, b, a])])
    with pytest.raises(JadeError):
        rt.execute([(k, [a, b, wrong])])
    with pytest.raises(JadeError):
        rt.execute([])
    with pytest.raises(JadeError):
        rt.execute([(k, [a, b, wrong])], repeats=0)


def test_ordering_ownership_alias(rt):
    # metal.rs:919-991
    other = jc.Runtime(0)
    try:
        a, b = resident(rt, np.array([0, 1, -2, 3, 1], np.float32)), resident(rt, np.array([-1, 2, 3, -4, 7], np.float32))
        mid, out = rt.alloc(5), rt.alloc(5)
        foreign = other.alloc(5)
        with pytest.raises(JadeError):
            rt.upload(a, np.ones(1, np.float32))
        with pytest.raises(JadeError):
            rt.upload(foreign, np.zeros(5, np.float32))
        add = rt.compile({"op": "add", "len": 5})
        foreign_add = other.compile({"op": "add", "len": 5})
        with pytest.raises(JadeError):
            rt.execute([(foreign_add, [a, b, out])])
        with pytest.raises(JadeError):
            rt.execute([(add, [a, b, a])])
        # a bad later job rejects the whole sequence before the first runs
        with pytest.raises(JadeError):
            rt.execute([(add, [a, b, mid]), (add, [mid, foreign, out])])
        assert rt.download(mid).tolist() == [0.0] * 5
        with pytest.raises(JadeError):
            rt.execute([(add, [a, b, mid]), (add, [mid, b, out])], repeats=0)
        t = rt.execute([(add, [a, b, mid]), (add, [mid, b, out])], repeats=3)
        assert t.dispatches == 6 and t.repeats == 3
        assert rt.download(out).tolist() == [-2, 5, 4, -5, 15]
        assert t.host_ms > 0 and (t.gpu_ms is None or t.gpu_ms > 0)
        # raw pointer not registered with this context is rejected natively too
        other_k = rt.compile({"op": "add", "len": 5})
        disp = (jc.runtime._Dispatch * 1)()
        arr = (ctypes.c_void_p * 3)(a.ptr, foreign.ptr, out.ptr)
        disp[0].kernel, disp[0].buffers, disp[0].buffer_count = other_k.handle, ctypes.cast(arr, ctypes.POINTER(ctypes.c_void_p)), 3
        e = ctypes.create_string_buffer(512)
        g = ctypes.c_double()
        assert jc.lib().jr_execute2(rt.ctx, disp, 1, 1, 0, ctypes.byref(g), None, e, 512) == JR_EINVAL
        assert b"another runtime" in e.value
    finally:
        other.close()


@pytest.mark.parametrize("gemm_op", ["gemm", "gemm_mps"])
def test_mixed_chain_ordering(rt, gemm_op):
    # metal.rs:827-916 (MPS -> shader -> MPS): here FP32 FFMA GEMM or the cuBLAS comparator
    spec = {"op": "gemm", "m": 2, "n": 2, "k": 2, "tiled": True} if gemm_op == "gemm" else \
        {"op": "gemm_mps", "m": 2, "n": 2, "k": 2}
    a = resident(rt, np.array([1, 2, 3, 4], np.float32))
    b = resident(rt, np.array([2, 0, 1, 2], np.float32))
    bias = resident(rt, np.array([1, -1, 2, -2], np.float32))
    ab = resident(rt, np.array([11, 12, 13, 14], np.float32))
    shifted, out = rt.alloc(4), rt.alloc(4)
    gemm, add = rt.compile(spec), rt.compile({"op": "add", "len": 4})
    other = jc.Runtime(0)
    try:
        foreign = other.alloc(4)
        with pytest.raises(JadeError):
            rt.execute([(gemm, [a, b, ab]), (add, [ab, foreign, shifted])])
        assert rt.download(ab).tolist() == [11, 12, 13, 14]
    finally:
        other.close()
    with pytest.raises(JadeError):
        rt.execute([(gemm, [a, b, a])])
    t = rt.execute([(gemm, [a, b, ab]), (add, [ab, bias, shifted]), (gemm, [shifted, b, out])], repeats=3)
    assert t.dispatches == 9
    assert rt.download(ab).tolist() == [4, 4, 10, 8]
    assert rt.download(shifted).tolist() == [5, 3, 12, 6]
    assert rt.download(out).tolist() == [13, 6, 30, 12]
    # read/read aliasing is valid (metal.rs:819-822)
    rt.execute([(gemm, [a, a, out])])
    assert rt.download(out).tolist() == [7, 10, 15, 22]


GEMM_SHAPES = [(1, 1, 1), (7, 9, 13), (8, 8, 8), (31, 47, 19), (32, 32, 33), (33, 31, 65), (65, 67, 63),
               (1, 129, 33), (64, 64, 64), (127, 65, 129), (256, 256, 65), (257, 263, 67),
               # K and N multiples of 4: the TMA-fed FFMA kernel (ragged M, N and k tiles)
               (1, 4, 4), (33, 36, 20), (100, 68, 132), (129, 260, 516), (300, 128, 1024), (1100, 1200, 36)]


@pytest.mark.parametrize("mnk", GEMM_SHAPES, ids=str)
def test_fp32_gemm_shapes_bit_exact(rt, mnk):
    # metal_lab.rs:400-413 shapes, inputs as metal_lab.rs:135-136
    m, n, k = mnk
    a, b = O.values(m * k, 0x1234, 1.0), O.values(k * n, 0xABCD, 1.0 / np.sqrt(np.float32(k)))
    got, _, kern = run(rt, {"op": "gemm", "m": m, "n": n, "k": k, "tiled": True}, [a, b])
    rc, r = O.compare(got, O.gemm_reference(m, n, k, a, b), 5e-5, 5e-5)
    assert rc == 0, r.max_abs_error
    assert np.array_equal(got, O.gemm_fp32_sequential(m, n, k, a, b))
    rc, v = O.validation_check(m, n, k, a, b, got)
    assert rc == 0 and v.max_scaled_error < 1


ATTN_CASES = [(1, 1, 1, False, 1.0, False), (1, 1, 128, True, 1.0, False), (2, 7, 17, False, 1.0, False),
              (2, 7, 17, True, 1.0, False), (2, 33, 64, False, 1.0, False), (2, 33, 64, True, 1.0, False),
              (1, 65, 128, True, 1.0, False), (3, 17, 33, False, 1.0, True), (2, 17, 31, True, 1.0, True),
              (2, 17, 64, False, 20.0, False), (2, 17, 64, True, 20.0, False)]


@pytest.mark.parametrize("case", ATTN_CASES, ids=str)
@pytest.mark.parametrize("path", ["online", "materialized"])
def test_fp32_attention_configs(rt, case, path):
    # metal_lab.rs:419-431 configs, inputs metal_lab.rs:276-286, tolerance :333
    h, s, d, causal, amp, zeros = case
    n = h * s * d
    q = np.zeros(n, np.float32) if zeros else O.values(n, 0x1111, amp)
    k = np.zeros(n, np.float32) if zeros else O.values(n, 0x2222, amp)
    v = O.values(n, 0x3333, 1.0)
    expected = O.attention(h, s, d, causal, q, k, v)
    tol = 5e-4 if amp > 1 else 5e-5
    if path == "online":
        got, _, _ = run(rt, {"op": "attention_online", "heads": h, "seq": s, "dim": d, "causal": causal}, [q, k, v])
    else:
        qb, kb, vb = resident(rt, q), resident(rt, k), resident(rt, v)
        scores, probs, out = rt.alloc(h * s * s), rt.alloc(h * s * s), rt.alloc(n)
        jobs = [(rt.compile({"op": "attention_scores", "heads": h, "seq": s, "dim": d, "causal": causal}), [qb, kb, scores]),
                (rt.compile({"op": "softmax", "rows": h * s, "cols": s}), [scores, probs]),
                (rt.compile({"op": "attention_apply", "heads": h, "seq": s, "dim": d}), [probs, vb, out])]
        rt.execute(jobs, repeats=2)
        got = rt.download(out)
        assert rt.download(qb).tolist() == q.tolist()  # inputs unmodified (metal_lab.rs:363-366)
    rc, r = O.compare(got, expected, tol, tol)
    assert rc == 0, (r.first_bad_index, r.max_abs_error)


@pytest.mark.parametrize("ab", [(1.0001, 1.0003), (70000.25, 1.0000312)])
@pytest.mark.parametrize("op", ["gemm", "gemm_simd", "gemm_mps"])
def test_fp32_precision_probes(rt, ab, op):
    # metal_lab.rs:436-461: no reduced precision anywhere in the FP32 path
    a, b = np.float32(ab[0]), np.float32(ab[1])
    spec = {"op": op, "m": 1, "n": 1, "k": 1}
    if op == "gemm":
        spec["tiled"] = True
    got, _, _ = run(rt, spec, [np.array([a]), np.array([b])], repeats=1)
    rc, _ = O.compare(got, np.array([float(a) * float(b)]), 1e-5, 1e-6)
    assert rc == 0


@pytest.mark.parametrize("rows,cols", [(1, 1), (3, 17), (7, 4096), (5, 8192), (2, 20000), (3, 65536 + 8)])
@pytest.mark.parametrize("dtype", ["fp32", "bf16"])
def test_row_kernels(rt, rows, cols, dtype):
    x = rt.alloc(rows * cols, dtype)
    w = rt.alloc(cols, dtype)
    rt.fill(x, "normal", seed=11, lo=0.0, hi=1.0)
    rt.fill(w, "uniform", seed=11, stream=1, lo=0.5, hi=1.5)
    xf, wf = rt.download_f32(x), rt.download_f32(w)
    y, p = rt.alloc(rows * cols, dtype), rt.alloc(rows * cols, dtype)
    inv = rt.alloc(rows)
    base = {"rows": rows, "cols": cols, "dtype": dtype}
    rt.execute([(rt.compile({"op": "rms_norm", "epsilon": 1e-6, **base}), [x, w, y]),
                (rt.compile({"op": "softmax", **base}), [x, p]),
                (rt.compile({"op": "rms_inv", "epsilon": 1e-6, **base}), [x, inv])])
    eps = float(np.float32(1e-6))
    tol = 3e-5 if dtype == "fp32" else 2 ** -8
    rc, r = O.compare(rt.download_f32(y), O.normalize(rows, cols, xf, wf, eps), tol, tol)
    assert rc == 0, r.max_abs_error
    rc, r = O.compare(rt.download_f32(p), O.softmax(rows, cols, 4 * xf / 4), tol, tol)
    assert rc == 0, r.max_abs_error
    X = xf.reshape(rows, cols).astype(np.float64)
    rc, _ = O.compare(rt.download(inv), 1 / np.sqrt((X * X).mean(1) + eps), 3e-5, 3e-5)
    assert rc == 0


STAGED, REGISTER = "row_staged_", "row_register_"


@pytest.mark.parametrize("rows,cols,dtype,paths", [(2000, 8192, "bf16", (STAGED,) * 3), (3001, 4096, "bf16", (STAGED,) * 3),
                                                   (700, 32768, "bf16", (STAGED,) * 3), (1500, 2048, "bf16", (STAGED,) * 3),
                                                   (2000, 8192, "fp32", (REGISTER, STAGED, REGISTER)),
                                                   (700, 16384, "fp32", (REGISTER,) * 3)])
def test_row_kernels_many_rows(rt, rows, cols, dtype, paths):
    # many rows per CTA: 16-bit rows and FP32 softmax rows up to 32 KB staged
    # through shared memory by bulk copies (several rows per ring position), the
    # other FP32 rows register-resident (the kernel name says which path ran;
    # paths = rms_norm, softmax, rms_inv)
    x = rt.alloc(rows * cols, dtype)
    w = rt.alloc(cols, dtype)
    rt.fill(x, "normal", seed=5, lo=0.0, hi=2.0)
    rt.fill(w, "uniform", seed=5, stream=1, lo=0.5, hi=1.5)
    xf, wf = rt.download_f32(x), rt.download_f32(w)
    y, p, inv = rt.alloc(rows * cols, dtype), rt.alloc(rows * cols, dtype), rt.alloc(rows)
    base = {"rows": rows, "cols": cols, "dtype": dtype}
    kerns = [rt.compile({"op": "rms_norm", "epsilon": 1e-6, **base}), rt.compile({"op": "softmax", **base}),
             rt.compile({"op": "rms_inv", "epsilon": 1e-6, **base})]
    for k, path in zip(kerns, paths):
        assert k.info["impl"].startswith(path), k.info
    rt.execute([(kerns[0], [x, w, y]), (kerns[1], [x, p]), (kerns[2], [x, inv])], repeats=2)
    eps = float(np.float32(1e-6))
    tol = 3e-5 if dtype == "fp32" else 2 ** -8
    rc, r = O.compare(rt.download_f32(y), O.normalize(rows, cols, xf, wf, eps), tol, tol)
    assert rc == 0, r.max_abs_error
    rc, r = O.compare(rt.download_f32(p), O.softmax(rows, cols, xf), tol, tol)
    assert rc == 0, r.max_abs_error
    X = xf.reshape(rows, cols).astype(np.float64)
    rc, _ = O.compare(rt.download(inv), 1 / np.sqrt((X * X).mean(1) + eps), 3e-5, 3e-5)
    assert rc == 0


def test_softmax_stress_rows(rt):
    # BASELINE config 3 scales logits by 4; extreme rows as workloads.rs:125-133
    rows, cols = 4, 8192
    i = np.arange(rows * cols)
    x = np.where(i // cols == 0, np.float32(1000.0), (i % cols).astype(np.float32) * np.float32(0.25) - np.float32(10000.0)).astype(np.float32)
    got, _, _ = run(rt, {"op": "softmax", "rows": rows, "cols": cols}, [x])
    rc, _ = O.compare(got, O.softmax(rows, cols, x), 3e-5, 3e-5)
    assert rc == 0


@pytest.mark.parametrize("n", [1, 3, 4, 257, 1 << 20, (1 << 20) + 5])
def test_elementwise_and_swiglu_sizes(rt, n):
    rng = np.random.default_rng(n)
    x = rng.uniform(-1, 1, n).astype(np.float32)
    y = rng.uniform(-1, 1, n).astype(np.float32)
    spec = {"op": "elementwise", "len": n, "inputs": 2, "expression": O._relu_expr()}
    got, _, _ = run(rt, spec, [x, y], repeats=1)
    assert np.array_equal(got, O.expr_eval_f32(spec["expression"], [x, y]))
    g = (rng.standard_normal(n) * 8).astype(np.float32)
    got, _, _ = run(rt, {"op": "swi_glu", "len": n}, [g, y], repeats=1)
    rc, _ = O.compare(got, O.swiglu(g, y), 3e-5, 3e-5)
    assert rc == 0
    gb, yb = rt.alloc(n, "bf16"), rt.alloc(n, "bf16")
    rt.upload(gb, jc.f32_to_bf16(g))
    rt.upload(yb, jc.f32_to_bf16(y))
    ob = rt.alloc(n, "bf16")
    rt.execute([(rt.compile({"op": "swi_glu", "len": n, "dtype": "bf16"}), [gb, yb, ob])])
    exp = O.swiglu(jc.bf16_to_f32(jc.f32_to_bf16(g)), jc.bf16_to_f32(jc.f32_to_bf16(y)))
    rc, _ = O.compare(rt.download_f32(ob), exp, 1e-3, 2 ** -8)
    assert rc == 0


def test_graph_replay_matches_stream_replay(rt):
    a = resident(rt, np.array([0, 1, -2, 3, 1], np.float32))
    b = resident(rt, np.array([-1, 2, 3, -4, 7], np.float32))
    mid, out = rt.alloc(5), rt.alloc(5)
    add = rt.compile({"op": "add", "len": 5})
    t = rt.execute([(add, [a, b, mid]), (add, [mid, b, out])], repeats=10, graph=True)
    assert rt.download(out).tolist() == [-2, 5, 4, -5, 15] and t.dispatches == 20


def test_per_job_timing_and_copy_jobs(rt):
    n = 1 << 22
    hin = rt.host_alloc(n)
    hout = rt.host_alloc(n)
    hin.host_view()[:] = np.arange(n, dtype=np.float32)
    d, e = rt.alloc(n), rt.alloc(n)
    h2d = rt.compile({"op": "copy", "bytes": 4 * n, "direction": "h2d"})
    d2h = rt.compile({"op": "copy", "bytes": 4 * n, "direction": "d2h"})
    add = rt.compile({"op": "add", "len": n})
    t = rt.execute([(h2d, [hin, d]), (add, [d, d, e]), (d2h, [e, hout])], repeats=2, per_job=True)
    assert np.array_equal(hout.host_view(), 2 * np.arange(n, dtype=np.float32))
    assert len(t.job_ms) == 3 and all(x > 0 for x in t.job_ms)
    with pytest.raises(JadeError):  # device buffer where a pinned host buffer is required
        rt.execute([(h2d, [d, e])])


def test_dependency_scheduled_streams_keep_order(rt):
    # JR_EXEC_STREAMS: transfers on their own streams, ordered by the data hazards
    # of their bindings only. Two rounds reuse the same device buffers, so every
    # kind of hazard appears: the second upload into d must wait for the first
    # add to read d (write after read), the second add into e for the first
    # read-back of e (write after read) and the read-backs for their adds (read
    # after write). 64 MB buffers make a violated order visible in the results.
    n = 1 << 24
    h1, h2, o1, o2 = (rt.host_alloc(n) for _ in range(4))
    h1.host_view()[:] = np.arange(n, dtype=np.float32)
    h2.host_view()[:] = -np.arange(n, dtype=np.float32) - 1
    d, e = rt.alloc(n), rt.alloc(n)
    h2d = rt.compile({"op": "copy", "bytes": 4 * n, "direction": "h2d"})
    d2h = rt.compile({"op": "copy", "bytes": 4 * n, "direction": "d2h"})
    add = rt.compile({"op": "add", "len": n})
    jobs = [(h2d, [h1, d]), (add, [d, d, e]), (d2h, [e, o1]), (h2d, [h2, d]), (add, [d, d, e]), (d2h, [e, o2])]
    for rep in range(3):
        o1.host_view()[:] = 0
        o2.host_view()[:] = 0
        t = rt.execute(jobs, repeats=2, streams=True, per_job=(rep == 2))
        assert np.array_equal(o1.host_view(), 2 * np.arange(n, dtype=np.float32))
        assert np.array_equal(o2.host_view(), -2 * np.arange(n, dtype=np.float32) - 2)
        assert t.gpu_ms > 0
    assert len(t.job_ms) == 6 and all(x > 0 for x in t.job_ms)
    with pytest.raises(JadeError, match="cannot be combined"):
        rt.execute(jobs, streams=True, graph=True)


def test_fill_is_deterministic_and_distributed(rt):
    n = 1 << 20
    a, b = rt.alloc(n), rt.alloc(n)
    rt.fill(a, "normal", seed=5, stream=2, lo=0.0, hi=1.0)
    rt.fill(b, "normal", seed=5, stream=2, lo=0.0, hi=1.0)
    x = rt.download(a)
    assert np.array_equal(x, rt.download(b))
    assert abs(x.mean()) < 0.01 and abs(x.std() - 1) < 0.01
    rt.fill(a, "uniform", seed=5, stream=3, lo=-1.0, hi=1.0)
    u = rt.download(a)
    assert u.min() >= -1 and u.max() < 1 and abs(u.mean()) < 0.01


REF_GEN = sorted(glob.glob(os.path.join(REF_BUILD, "generated", "*.so")))


def abi1(L):
    """ctypes signatures of native/jade_runtime_corex.h:18-31."""
    vp, sz, cp, i32, u32 = ctypes.c_void_p, ctypes.c_size_t, ctypes.c_char_p, ctypes.c_int, ctypes.c_uint32
    L.jr_version.restype = u32
    L.jr_create.argtypes = [i32, ctypes.POINTER(vp), cp, sz]
    L.jr_destroy.argtypes = [vp]
    L.jr_destroy.restype = None
    L.jr_info.argtypes = [vp, cp, sz, cp, sz]
    L.jr_alloc.argtypes = [vp, sz, ctypes.POINTER(vp), cp, sz]
    L.jr_free.argtypes = [vp, vp]
    L.jr_free.restype = None
    L.jr_upload.argtypes = [vp, vp, vp, sz, cp, sz]
    L.jr_download.argtypes = [vp, vp, vp, sz, cp, sz]
    L.jr_execute.argtypes = [vp, vp, sz, u32, ctypes.POINTER(ctypes.c_double), cp, sz]
    return L


@pytest.mark.skipif(not REF_GEN, reason="reference emitted kernels not built (oracle/_ref)")
@pytest.mark.parametrize("case", O.conformance_cases(), ids=lambda c: c[0])
def test_abi1_reference_modules_match_builtin(rt, case):
    """Runs the reference's own emitted CUDA module for the case (compiled from
    reports/generated-native into oracle/_ref) through this library's ABI-1
    jr_execute, and compares with the built-in sm_100a kernel's output."""
    name, spec, inputs, expected = case

    def run_module(directory):
        mod = ctypes.CDLL(os.path.join(REF_BUILD, directory, name + ".so"))
        bufs = [resident(rt, x) for x in inputs]
        out = rt.alloc(len(expected))
        arr = (ctypes.c_void_p * (len(bufs) + 1))(*[b.ptr for b in bufs], out.ptr)
        job = (ctypes.c_void_p * 3)(ctypes.cast(mod.jade_generated_launch, ctypes.c_void_p).value,
                                    ctypes.cast(arr, ctypes.c_void_p).value, len(bufs) + 1)
        e = ctypes.create_string_buffer(512)
        g = ctypes.c_double()
        assert jc.lib().jr_execute(rt.ctx, job, 1, 2, ctypes.byref(g), e, 512) == 0, e.value
        return rt.download(out)

    ref_out = run_module("generated")
    mine, _, _ = run(rt, spec, inputs)
    rc, _ = O.compare(ref_out, expected, 3e-5, 3e-5)
    assert rc == 0
    op = spec["op"]
    if op in ("axpy", "add", "gemm", "swi_glu"):
        assert np.array_equal(mine, ref_out), name  # same operation order -> same bits
    elif op == "elementwise" and not O.expr_has_exp(spec["expression"]):
        # nvcc contracts the emitted a*b+c into one FMA by default; with contraction
        # off the reference module and this backend agree bit for bit.
        nofma = os.path.join(REF_BUILD, "generated_nofma", name + ".so")
        if os.path.exists(nofma):
            assert np.array_equal(mine, run_module("generated_nofma")), name
        rc, _ = O.compare(mine, ref_out.astype(np.float64), 3e-5, 3e-5)
        assert rc == 0
    else:
        rc, _ = O.compare(mine, ref_out.astype(np.float64), 3e-5, 3e-5)
        assert rc == 0


@pytest.mark.skipif(not os.path.exists(os.path.join(REF_BUILD, "libjade_runtime_corex.so")) or not REF_GEN,
                    reason="reference bridge not built (oracle/_ref)")
def test_reference_bridge_and_this_library_agree_on_abi1():
    """The same ABI-1 call sequence through the reference's bridge
    (native/jade_runtime_corex.cpp built in oracle/_ref) and through this library."""
    results = []
    for path in (os.path.join(REF_BUILD, "libjade_runtime_corex.so"), jc.library_path()):
        L = abi1(ctypes.CDLL(path))
        assert L.jr_version() == 1
        ctx = ctypes.c_void_p()
        e = ctypes.create_string_buffer(1024)
        assert L.jr_create(0, ctypes.byref(ctx), e, 1024) == 0, e.value
        info = ctypes.create_string_buffer(2048)
        assert L.jr_info(ctx, info, 2048, e, 1024) == 0
        assert info.value.startswith(b"device=0 name=")
        name, spec, inputs, expected = O.conformance_cases()[4]  # add_257
        mod = ctypes.CDLL(os.path.join(REF_BUILD, "generated", name + ".so"))
        ptrs = []
        for x in inputs + [np.zeros(len(expected), np.float32)]:
            p = ctypes.c_void_p()
            assert L.jr_alloc(ctx, x.nbytes, ctypes.byref(p), e, 1024) == 0
            assert L.jr_upload(ctx, p, ctypes.c_void_p(x.ctypes.data), x.nbytes, e, 1024) == 0
            ptrs.append(p.value)
        arr = (ctypes.c_void_p * len(ptrs))(*ptrs)
        job = (ctypes.c_void_p * 3)(ctypes.cast(mod.jade_generated_launch, ctypes.c_void_p).value,
                                    ctypes.cast(arr, ctypes.c_void_p).value, len(ptrs))
        g = ctypes.c_double()
        assert L.jr_execute(ctx, job, 1, 3, ctypes.byref(g), e, 1024) == 0
        assert g.value >= 0
        # rejected calls: empty list, zero repeats, null buffer
        assert L.jr_execute(ctx, job, 0, 1, ctypes.byref(g), e, 1024) == 1
        assert L.jr_execute(ctx, job, 1, 0, ctypes.byref(g), e, 1024) == 1
        out = np.empty(len(expected), np.float32)
        assert L.jr_download(ctx, ctypes.c_void_p(ptrs[-1]), ctypes.c_void_p(out.ctypes.data), out.nbytes, e, 1024) == 0
        for p in ptrs:
            L.jr_free(ctx, ctypes.c_void_p(p))
        L.jr_destroy(ctx)
        results.append(out)
    assert np.array_equal(results[0], results[1])


def test_fp32_ffma_gemm_baseline_config1_bit_exact(rt):
    # FP32 C = A.B, M = N = K = 512, A and B ~ U[-1,1] from seed
    # 0, FP32 accumulation. The FFMA kernel sums the k products in order with one
    # fmaf each, so it equals the sequential FP32 oracle bit for bit, and it is
    # within validation.rs:35-91 of the FP64 oracle (north_star: <= 1e-5 relative).
    m = n = k = 512
    a, b = rt.alloc(m * k), rt.alloc(k * n)
    rt.fill(a, "uniform", seed=0, stream=0, lo=-1.0, hi=1.0)
    rt.fill(b, "uniform", seed=0, stream=1, lo=-1.0, hi=1.0)
    out = rt.alloc(m * n)
    kern = rt.compile({"op": "gemm", "m": m, "n": n, "k": k, "tiled": True})
    assert kern.info["path"] == "simt", kern.info
    rt.execute([(kern, [a, b, out])])
    af, bf, got = rt.download(a), rt.download(b), rt.download(out)
    assert np.array_equal(got, O.gemm_fp32_sequential(m, n, k, af, bf, threads=O.max_threads()))
    rc, v = O.validation_check(m, n, k, af, bf, got)
    assert rc == 0 and v.max_scaled_error < 1
    print(f"C1 FFMA 512^3: bit-exact to the sequential FP32 sum; max |err|/sum|a*b| vs FP64 = {v.max_magnitude_error:.2e}")


@pytest.fixture(scope="module")
def emitted_modules(tmp_path_factory):
    """Every conformance case emitted for the "cuda" target (jr_spec_emit) and
    built with nvcc for sm_100a, as a user of `jade-runtime emit` would."""
    import concurrent.futures
    import shutil
    import subprocess
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(nvcc):
        pytest.skip("nvcc not available")
    out = tmp_path_factory.mktemp("emitted")

    def build(case):
        name, spec = case[0], case[1]
        src = out / f"{name}.cu"
        src.write_text(jc.emit(spec, "cuda"))
        r = subprocess.run([nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-shared", "-Xcompiler", "-fPIC",
                            "-o", str(out / f"{name}.so"), str(src)], capture_output=True, text=True, timeout=300)
        assert r.returncode == 0, (name, r.stderr[-2000:])
        return name, str(out / f"{name}.so")

    with concurrent.futures.ThreadPoolExecutor(8) as ex:
        return dict(ex.map(build, O.conformance_cases()))


@pytest.mark.parametrize("case", O.conformance_cases(), ids=lambda c: c[0])
def test_abi1_emitted_cuda_modules(rt, emitted_modules, case):
    """The sm_100a module emitted for the case (`emit --target cuda`) runs through
    ABI-1 jr_execute like the reference's generated modules: bit-exact with the
    built-in kernel where both fix the operation order (elementwise trees, axpy,
    add, SwiGLU, k-ordered GEMM), within the reference's 3e-5 of the FP64 oracle
    for the row reductions."""
    name, spec, inputs, expected = case
    mod = ctypes.CDLL(emitted_modules[name])
    bufs = [resident(rt, x) for x in inputs]
    out = rt.alloc(len(expected))
    arr = (ctypes.c_void_p * (len(bufs) + 1))(*[b.ptr for b in bufs], out.ptr)
    job = (ctypes.c_void_p * 3)(ctypes.cast(mod.jade_generated_launch, ctypes.c_void_p).value,
                                ctypes.cast(arr, ctypes.c_void_p).value, len(bufs) + 1)
    e = ctypes.create_string_buffer(512)
    g = ctypes.c_double()
    assert jc.lib().jr_execute(rt.ctx, job, 1, 2, ctypes.byref(g), e, 512) == 0, e.value
    got = rt.download(out)
    rc, r = O.compare(got, expected, 3e-5, 3e-5)
    assert rc == 0, (name, r.first_bad_index, r.max_abs_error)
    if spec["op"] in ("axpy", "add", "gemm", "swi_glu", "elementwise"):
        mine, _, _ = run(rt, spec, inputs)
        assert np.array_equal(mine, got), name


@pytest.mark.parametrize("dtype", ["fp32", "bf16"])
@pytest.mark.parametrize("cols", [256, 1024, 8192])
def test_softmax_rows_with_masked_scores(rt, dtype, cols):
    # causal-masked score rows (as attention_scores writes them): row r keeps its
    # first r+1 entries and holds -inf after them, so most threads of a row see
    # only -inf and must contribute e^-inf = 0, not NaN
    rows = 64
    x = np.random.default_rng(cols).standard_normal((rows, cols)).astype(np.float32) * 4
    keep = np.minimum(np.arange(rows) * (cols // rows) + 1, cols)
    x[np.arange(cols)[None, :] >= keep[:, None]] = -np.inf
    buf = rt.alloc(rows * cols, dtype)
    rt.upload(buf, x.ravel() if dtype == "fp32" else jc.runtime.f32_to_bf16(x.ravel()))
    out = rt.alloc(rows * cols, dtype)
    k = rt.compile({"op": "softmax", "rows": rows, "cols": cols, "dtype": dtype})
    rt.execute([(k, [buf, out])])
    got = rt.download_f32(out)
    assert np.isfinite(got).all()
    exp = O.softmax(rows, cols, rt.download_f32(buf))
    tol = (3e-5, 3e-5) if dtype == "fp32" else (2e-3, 2.0 ** -8)
    rc, r = O.compare(got, exp, *tol)
    assert rc == 0, (r.first_bad_index, r.max_abs_error)
