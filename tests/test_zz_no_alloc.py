"""The allocation-free TF32 GEMM entry point (jr_gemm_tf32_kn_noalloc).

It exists for callers that cannot allocate device memory at call time (a host
framework that owns every device allocation through its own pool, or a
latency-critical loop where cudaMalloc's implicit synchronisation is not
acceptable); its scratch is a static 16 MiB array inside the library. This test
calls it through the C ABI twice in a row and checks each result against the
compiled entry point (jr_compile + jr_execute2 of the same GEMM spec), within
this suite's TF32 tolerance (src/validation.rs:35-91 form, reduced-precision
coefficient 0.0012). The compiled GEMM is built with split-K off
(JADE_GEMM_SPLIT_K=1), so that both entry points sum each output's K products
in the same order, as this entry point always does. The file name makes pytest
collect it last.
"""
import ctypes

import numpy as np
import pytest

import jade_compute_b200 as jc
from oracle import oracle as O

pytestmark = pytest.mark.gpu

SCRATCH_ELEMENTS = 4 << 20  # K*N limit of the static scratch (16 MiB of FP32)


def noalloc_fn():
    f = jc.lib().jr_gemm_tf32_kn_noalloc
    f.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_uint32, ctypes.c_uint32,
                  ctypes.c_uint32, ctypes.c_void_p, ctypes.c_char_p, ctypes.c_size_t]
    f.restype = ctypes.c_int
    return f


def operands(rt, m, n, k, seed):
    a, b = rt.alloc(m * k, "tf32"), rt.alloc(k * n, "tf32")
    rt.fill(a, "uniform", seed=seed, stream=0, lo=-1.0, hi=1.0)
    rt.fill(b, "uniform", seed=seed, stream=1, lo=-1.0, hi=1.0)
    return a, b


def test_noalloc_matches_compiled_entry_point_twice(monkeypatch):
    monkeypatch.setenv("JADE_GEMM_SPLIT_K", "1")  # one K range, as in this entry point
    f = noalloc_fn()
    rt = jc.Runtime(0)
    try:
        # large then small, and the exact K*N = 4,194,304 limit (K=1024, N=4096)
        for call, (m, n, k) in enumerate([(384, 1024, 2048), (200, 300, 136), (256, 4096, 1024)]):
            assert k * n <= SCRATCH_ELEMENTS
            a, b = operands(rt, m, n, k, 40 + call)
            ref_out, out = rt.alloc(m * n), rt.alloc(m * n)
            kern = rt.compile({"op": "gemm", "m": m, "n": n, "k": k, "tiled": True, "dtype": "tf32"})
            rt.execute([(kern, [a, b, ref_out])])
            err = ctypes.create_string_buffer(256)
            rc = f(a.ptr, b.ptr, out.ptr, m, n, k, None, err, 256)
            assert rc == 0, err.value
            got, want = rt.download(out), rt.download(ref_out)
            af, bf = rt.download(a), rt.download(b)
            rc1, v = O.validation_check(m, n, k, af, bf, got, budget=1 << 14, fp16=True)
            assert rc1 == 0, v.max_scaled_error
            rc2, r = O.compare(got, want.astype(np.float64), 1e-4, 1e-4)
            assert rc2 == 0, r.max_abs_error
            print(f"noalloc {m}x{n}x{k}: max scaled error {v.max_scaled_error:.3e}, "
                  f"max |noalloc - compiled| {r.max_abs_error:.3e}")
    finally:
        rt.close()


def test_noalloc_ragged_n_against_oracle():
    # N % 4 != 0: the epilogue's scalar tail, B transposed through the static
    # scratch; the compiled [K,N] TF32 path refuses this N, so the FP64 oracle
    # is the only check
    f = noalloc_fn()
    rt = jc.Runtime(0)
    try:
        m, n, k = 64, 302, 136
        a, b = operands(rt, m, n, k, 77)
        out = rt.alloc(m * n)
        err = ctypes.create_string_buffer(256)
        for _ in range(2):
            assert f(a.ptr, b.ptr, out.ptr, m, n, k, None, err, 256) == 0, err.value
            rc, v = O.validation_check(m, n, k, rt.download(a), rt.download(b), rt.download(out), fp16=True)
            assert rc == 0, (v.first_bad_index, v.max_scaled_error)
    finally:
        rt.close()


def test_noalloc_allocates_nothing():
    import torch
    f = noalloc_fn()
    rt = jc.Runtime(0)
    try:
        m, n, k = 256, 512, 512
        a, b = operands(rt, m, n, k, 5)
        out = rt.alloc(m * n)
        err = ctypes.create_string_buffer(256)
        torch.cuda.mem_get_info(0)  # the query's own context set-up happens here
        assert f(a.ptr, b.ptr, out.ptr, m, n, k, None, err, 256) == 0, err.value  # first call: set-up
        free_before = torch.cuda.mem_get_info(0)[0]
        for _ in range(3):
            assert f(a.ptr, b.ptr, out.ptr, m, n, k, None, err, 256) == 0, err.value
        assert torch.cuda.mem_get_info(0)[0] == free_before
    finally:
        rt.close()


def test_noalloc_rejects_oversized_and_unaligned():
    f = noalloc_fn()
    rt = jc.Runtime(0)
    try:
        a, b, c = rt.alloc(16), rt.alloc(16), rt.alloc(16)
        err = ctypes.create_string_buffer(256)
        assert f(a.ptr, b.ptr, c.ptr, 1, 4096, 4096, None, err, 256) == 1  # k*n = 16 Mi > 4 Mi elements
        assert b"static scratch" in err.value
        assert f(a.ptr, b.ptr, c.ptr, 1, 4097, 1024, None, err, 256) == 1  # one column past the limit
        assert b"static scratch" in err.value
        assert f(a.ptr, b.ptr, c.ptr, 4, 4, 3, None, err, 256) == 1  # k not a multiple of 4
        assert f(None, b.ptr, c.ptr, 4, 4, 4, None, err, 256) == 1
        assert f(a.ptr, b.ptr, c.ptr + 4, 1, 4, 4, None, err, 256) == 1  # out not 16-byte aligned
        assert b"out must be 16-byte aligned" in err.value
    finally:
        rt.close()
