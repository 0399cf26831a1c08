"""The fixed-shape GEMM plan ABI (include/jade_corex.h), the drop-in for the
reference's cuBLAS provider (native/jade_corex.h / jade_corex.cpp:110-266, loaded
by src/corex.rs:55-84).

CPU: every declared symbol is exported, the ABI version, and the host-side
validation (codes and messages of jade_corex.cpp:113-119,185-188,207-211,234-236).
GPU: the reference's GEMM KAT (validation.rs:102-112: a=[1,2,-3,4], b=[1..6] ->
[9,12,15,13,14,15]) in both precisions; parity with the FP64 oracle on the
reference's validation inputs (validation.rs:5-21) - FP32 bit-exact against the
k-ordered FP32 oracle, FP16 inputs within the validation.rs:35-91 bound evaluated
on the FP16-rounded inputs (the reference's own FP16 oracle, main.rs:166-172);
and the state machine (upload before run, run before download).
"""
import ctypes
import re

import numpy as np
import pytest

import jade_compute_b200 as jc
from oracle import oracle as O

HEADER = jc.runtime.INCLUDE.replace("jade_runtime.h", "jade_corex.h")


def lib():
    L = ctypes.CDLL(jc.library_path())
    L.jade_corex_abi_version.restype = ctypes.c_uint32
    L.jade_corex_create.argtypes = [ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_int, ctypes.c_uint32,
                                    ctypes.POINTER(ctypes.c_void_p), ctypes.c_char_p, ctypes.c_size_t]
    fp = ctypes.POINTER(ctypes.c_float)
    L.jade_corex_upload.argtypes = [ctypes.c_void_p, fp, ctypes.c_size_t, fp, ctypes.c_size_t, ctypes.c_char_p,
                                    ctypes.c_size_t]
    L.jade_corex_run.argtypes = [ctypes.c_void_p, ctypes.c_uint32, ctypes.POINTER(ctypes.c_double), ctypes.c_char_p,
                                 ctypes.c_size_t]
    L.jade_corex_download.argtypes = [ctypes.c_void_p, fp, ctypes.c_size_t, ctypes.c_char_p, ctypes.c_size_t]
    L.jade_corex_device_info.argtypes = [ctypes.c_void_p, ctypes.c_char_p, ctypes.c_size_t, ctypes.c_char_p,
                                         ctypes.c_size_t]
    L.jade_corex_destroy.argtypes = [ctypes.c_void_p]
    return L


def fptr(a):
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_float))


class Plan:
    def __init__(self, m, n, k, precision, device=0):
        self.L, self.m, self.n, self.k = lib(), m, n, k
        self.h = ctypes.c_void_p()
        self.err = ctypes.create_string_buffer(512)
        rc = self.L.jade_corex_create(m, n, k, device, precision, ctypes.byref(self.h), self.err, 512)
        assert rc == 0, self.err.value

    def upload(self, a, b):
        a = np.ascontiguousarray(a, np.float32)
        b = np.ascontiguousarray(b, np.float32)
        return self.L.jade_corex_upload(self.h, fptr(a), a.size, fptr(b), b.size, self.err, 512)

    def run(self, iterations=1):
        ms = ctypes.c_double(-1)
        rc = self.L.jade_corex_run(self.h, iterations, ctypes.byref(ms), self.err, 512)
        return rc, ms.value

    def download(self, count=None):
        out = np.zeros(count if count is not None else self.m * self.n, np.float32)
        rc = self.L.jade_corex_download(self.h, fptr(out), out.size, self.err, 512)
        return rc, out

    def close(self):
        self.L.jade_corex_destroy(self.h)


def test_plan_abi_exports_and_version():
    names = re.findall(r"^JC_API [a-z0-9_ *]+?\b(jade_corex\w+)\(", open(HEADER).read(), re.M)
    assert sorted(names) == sorted(["jade_corex_abi_version", "jade_corex_create", "jade_corex_upload", "jade_corex_run",
                                    "jade_corex_download", "jade_corex_device_info", "jade_corex_destroy"])
    L = lib()
    for n in names:
        assert hasattr(L, n), n
    assert L.jade_corex_abi_version() == 1
    L.jade_corex_destroy(None)  # null-safe


def test_plan_create_rejects_like_the_reference():
    L = lib()
    h = ctypes.c_void_p()
    e = ctypes.create_string_buffer(256)
    msg = b"dimensions must be 1..INT_MAX; device >= 0; precision 0 or 1"
    for args in [(0, 2, 2, 0, 0), (2, 0, 2, 0, 0), (2, 2, 0, 0, 0), (2, 2, 2, -1, 0), (2, 2, 2, 0, 2), (2**31, 2, 2, 0, 0)]:
        assert L.jade_corex_create(*args, ctypes.byref(h), e, 256) == 1
        assert e.value == msg and not h.value
    assert L.jade_corex_create(2, 2, 2, 0, 0, None, e, 256) == 1 and e.value == b"null output handle"
    assert L.jade_corex_create(2, 2, 2, 1000, 0, ctypes.byref(h), e, 256) == 1
    assert re.match(rb"device 1000 outside detected count \d+", e.value)
    # calls on a null context
    out = np.zeros(4, np.float32)
    assert L.jade_corex_upload(None, fptr(out), 4, fptr(out), 4, e, 256) == 1
    ms = ctypes.c_double()
    assert L.jade_corex_run(None, 1, ctypes.byref(ms), e, 256) == 1
    assert L.jade_corex_download(None, fptr(out), 4, e, 256) == 1
    assert L.jade_corex_device_info(None, e, 256, e, 256) == 1


@pytest.mark.gpu
@pytest.mark.parametrize("precision", [0, 1])
def test_plan_kat_and_state_machine(precision):
    p = Plan(2, 3, 2, precision)
    try:
        assert p.run()[0] == 1 and p.err.value == b"upload A/B before running"
        assert p.upload(np.zeros(3), np.zeros(6)) == 1
        assert p.err.value == b"upload requires non-null buffers and exact A/B element counts"
        assert p.upload([1, 2, -3, 4], [1, 2, 3, 4, 5, 6]) == 0
        assert p.download()[0] == 1 and p.err.value == b"run successfully before downloading C"
        assert p.run(0)[0] == 1
        rc, ms = p.run(3)
        assert rc == 0 and ms > 0, p.err.value
        assert p.download(5)[0] == 1 and p.err.value == b"download requires exact C element count"
        rc, out = p.download()
        assert rc == 0 and out.tolist() == [9, 12, 15, 13, 14, 15]
        info = ctypes.create_string_buffer(1024)
        assert p.L.jade_corex_device_info(p.h, info, 1024, p.err, 512) == 0
        s = info.value.decode()
        for key in ("device=0 ", "name=", "memory_bytes=", "multiprocessors=", "runtime_api=", "driver_api=", "blas_api=0",
                    "precision=" + ("fp16_inputs_fp32_accum_output" if precision else "fp32"), "kernel="):
            assert key in s, s
        assert p.L.jade_corex_device_info(p.h, info, 8, p.err, 512) == 1
        # a new upload invalidates the previous result
        assert p.upload([1, 2, -3, 4], [1, 2, 3, 4, 5, 6]) == 0 and p.download()[0] == 1
    finally:
        p.close()


def fp16_round(x):
    return np.asarray(x, np.float32).astype(np.float16).astype(np.float32)


@pytest.mark.gpu
@pytest.mark.parametrize("precision", [0, 1], ids=["fp32", "fp16"])
@pytest.mark.parametrize("mnk", [(1, 1, 1), (1, 17, 33), (17, 1, 35), (31, 47, 19), (64, 64, 64), (65, 33, 17),
                                 (3, 5, 257), (256, 384, 512), (1024, 1024, 1024)], ids=str)
def test_plan_parity(precision, mnk):
    # shapes of the reference's cuBLAS validation (main.rs:250-276) plus tensor-core sizes
    m, n, k = mnk
    a, b = O.validation_inputs(m, n, k)
    p = Plan(m, n, k, precision)
    try:
        assert p.upload(a, b) == 0, p.err.value
        rc, ms = p.run(2)
        assert rc == 0, p.err.value
        rc, got = p.download()
        assert rc == 0, p.err.value
    finally:
        p.close()
    if precision == 0:
        assert np.array_equal(got, O.gemm_fp32_sequential(m, n, k, a, b)), "FP32 plan is not the k-ordered FP32 sum"
    else:
        af, bf = fp16_round(a), fp16_round(b)
        rc, v = O.validation_check(m, n, k, af, bf, got)
        assert rc == 0, (rc, v.first_bad_index, v.max_scaled_error)
