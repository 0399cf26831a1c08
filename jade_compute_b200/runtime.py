"""Python host mirror of the reference's runtime contract over the C ABI.

The reference's Rust host (src/runtime/mod.rs:45-61 ``trait Runtime``;
src/runtime/corex.rs:335-613 ``impl Runtime for CorexRuntime``) owns buffers,
performs exact transfers, compiles validated KernelSpecs and executes ordered
batches. This module exposes the same operations (``info``, ``alloc``,
``upload``, ``download``, ``compile``, ``execute``) with the same argument
meaning and error behaviour, calling ``libjade_runtime.so`` through ctypes.
There is no CPU fallback: if the CUDA library is missing, importing the
runtime raises.
"""
from __future__ import annotations

import ctypes
import json
import os
import time
from dataclasses import dataclass, field
from typing import Iterable, Sequence

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
# JADE_RUNTIME_LIBRARY selects another build of this library (e.g. a variant
# compiled with different options); by default the in-tree build.
LIB_PATH = os.environ.get("JADE_RUNTIME_LIBRARY") or os.path.join(HERE, "lib", "libjade_runtime.so")
INCLUDE = os.path.join(os.path.dirname(HERE), "include", "jade_runtime.h")

JR_OK, JR_EINVAL, JR_ECUDA, JR_ENOMEM, JR_ETIMEOUT = 0, 1, 2, 3, 4
JR_EXEC_GRAPH = 1
JR_EXEC_STREAMS = 2

DTYPE_SIZE = {"fp32": 4, "tf32": 4, "bf16": 2, "fp16": 2, "u8": 1}
NP_DTYPE = {"fp32": np.float32, "tf32": np.float32, "bf16": np.uint16, "fp16": np.float16, "u8": np.uint8}


class JadeError(RuntimeError):
    """Error returned by the native runtime; ``code`` is the jr_* error code."""

    def __init__(self, code: int, message: str):
        super().__init__(f"Jade runtime error {code}: {message}")
        self.code = code
        self.message = message


_lib = None


def library_path() -> str:
    return LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"{LIB_PATH} is missing: build the CUDA extension first (__graft_entry__.build())")
    L = ctypes.CDLL(LIB_PATH, mode=ctypes.RTLD_GLOBAL)
    c_char_p, sz, vp, i32, u32 = ctypes.c_char_p, ctypes.c_size_t, ctypes.c_void_p, ctypes.c_int, ctypes.c_uint32
    u64p = ctypes.POINTER(ctypes.c_uint64)
    L.jr_version.restype = u32
    L.jr2_version.restype = u32
    L.jr_device_count.restype = i32
    L.jr_create.argtypes = [i32, ctypes.POINTER(vp), c_char_p, sz]
    L.jr_destroy.argtypes = [vp]
    L.jr_destroy.restype = None
    L.jr_info.argtypes = [vp, c_char_p, sz, c_char_p, sz]
    L.jr_alloc.argtypes = [vp, sz, ctypes.POINTER(vp), c_char_p, sz]
    L.jr_free.argtypes = [vp, vp]
    L.jr_free.restype = None
    L.jr_upload.argtypes = [vp, vp, vp, sz, c_char_p, sz]
    L.jr_download.argtypes = [vp, vp, vp, sz, c_char_p, sz]
    L.jr_execute.argtypes = [vp, vp, sz, u32, ctypes.POINTER(ctypes.c_double), c_char_p, sz]
    L.jr_spec_validate.argtypes = [c_char_p, c_char_p, sz]
    L.jr_spec_bindings.argtypes = [c_char_p, c_char_p, sz, c_char_p, sz]
    L.jr_spec_validate_bindings.argtypes = [c_char_p, u64p, u64p, sz, c_char_p, sz]
    L.jr_spec_launch.argtypes = [c_char_p, c_char_p, sz, c_char_p, sz]
    L.jr_spec_emit.argtypes = [c_char_p, c_char_p, c_char_p, sz, ctypes.POINTER(sz), c_char_p, sz]
    L.jr_spec_canonical.argtypes = [c_char_p, c_char_p, sz, c_char_p, sz]
    L.jr_compile.argtypes = [vp, c_char_p, ctypes.POINTER(vp), c_char_p, sz]
    L.jr_kernel_release.argtypes = [vp]
    L.jr_kernel_release.restype = None
    L.jr_kernel_info.argtypes = [vp, c_char_p, sz, c_char_p, sz]
    L.jr_execute2.argtypes = [vp, vp, sz, u32, u32, ctypes.POINTER(ctypes.c_double),
                              ctypes.POINTER(ctypes.c_double), c_char_p, sz]
    L.jr_buffer_bytes.argtypes = [vp, vp, ctypes.POINTER(sz)]
    L.jr_host_alloc.argtypes = [vp, sz, ctypes.POINTER(vp), c_char_p, sz]
    L.jr_host_free.argtypes = [vp, vp]
    L.jr_host_free.restype = None
    L.jr_comm_unique_id.argtypes = [ctypes.c_char_p, c_char_p, sz]
    L.jr_comm_init.argtypes = [vp, i32, i32, ctypes.c_char_p, u32, c_char_p, sz]
    L.jr_comm_init_all.argtypes = [ctypes.POINTER(vp), i32, u32, c_char_p, sz]
    L.jr_comm_destroy.argtypes = [vp]
    L.jr_peer_handle.argtypes = [vp, vp, ctypes.c_char_p, c_char_p, sz]
    L.jr_peer_attach.argtypes = [vp, vp, ctypes.c_char_p, i32, i32, c_char_p, sz]
    _lib = L
    return L


def _err():
    return ctypes.create_string_buffer(1024)


def _check(rc: int, err) -> None:
    if rc != JR_OK:
        raise JadeError(rc, err.value.decode(errors="replace"))


def _spec_text(spec) -> bytes:
    if isinstance(spec, (bytes, bytearray)):
        return bytes(spec)
    if isinstance(spec, str):
        return spec.encode()
    return json.dumps(spec).encode()


# ---------------------------------------------------------------- IR front end
def device_count() -> int:
    return lib().jr_device_count()


def spec_validate(spec) -> None:
    e = _err()
    _check(lib().jr_spec_validate(_spec_text(spec), e, len(e)), e)


def spec_bindings(spec) -> list:
    e, out = _err(), ctypes.create_string_buffer(1 << 16)
    _check(lib().jr_spec_bindings(_spec_text(spec), out, len(out), e, len(e)), e)
    return json.loads(out.value)


def spec_validate_bindings(spec, lengths: Sequence[int], ids: Sequence[int]) -> None:
    e = _err()
    n = len(lengths)
    L = (ctypes.c_uint64 * max(n, 1))(*lengths)
    I = (ctypes.c_uint64 * max(len(ids), 1))(*ids)
    if len(ids) != n:
        raise JadeError(JR_EINVAL, "lengths and ids differ in count")
    _check(lib().jr_spec_validate_bindings(_spec_text(spec), L, I, n, e, len(e)), e)


def spec_launch(spec) -> dict:
    e, out = _err(), ctypes.create_string_buffer(4096)
    _check(lib().jr_spec_launch(_spec_text(spec), out, len(out), e, len(e)), e)
    return json.loads(out.value)


def emit(spec, target: str = "corex") -> str:
    e = _err()
    need = ctypes.c_size_t(0)
    out = ctypes.create_string_buffer(1 << 16)
    rc = lib().jr_spec_emit(_spec_text(spec), target.encode(), out, len(out), ctypes.byref(need), e, len(e))
    if rc != JR_OK and need.value > len(out):
        out = ctypes.create_string_buffer(need.value)
        rc = lib().jr_spec_emit(_spec_text(spec), target.encode(), out, len(out), ctypes.byref(need), e, len(e))
    _check(rc, e)
    return out.value.decode()


def canonical(spec) -> str:
    e, out = _err(), ctypes.create_string_buffer(1 << 16)
    _check(lib().jr_spec_canonical(_spec_text(spec), out, len(out), e, len(e)), e)
    return out.value.decode()


# ---------------------------------------------------------------- bf16 helpers
def f32_to_bf16(x) -> np.ndarray:
    """Round-to-nearest-even FP32 -> BF16 bit patterns (uint16)."""
    b = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    nan = (b & 0x7F800000) == 0x7F800000
    nan &= (b & 0x7FFFFF) != 0
    r = ((b + 0x7FFF + ((b >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = ((b[nan] >> 16) | 0x40).astype(np.uint16)
    return r


def bf16_to_f32(h) -> np.ndarray:
    return (np.ascontiguousarray(h, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


# ---------------------------------------------------------------- objects
@dataclass
class Buffer:
    """Owned device (or pinned host) allocation. ``elements`` counts ``dtype`` items."""
    runtime: "Runtime"
    ptr: int
    nbytes: int
    dtype: str
    host: bool = False
    freed: bool = False

    @property
    def elements(self) -> int:
        return self.nbytes // DTYPE_SIZE[self.dtype]

    def __len__(self) -> int:
        return self.elements

    def free(self) -> None:
        if not self.freed and self.runtime.ctx:
            (lib().jr_host_free if self.host else lib().jr_free)(self.runtime.ctx, self.ptr)
        self.freed = True

    def host_view(self) -> np.ndarray:
        """numpy view of a pinned host buffer."""
        if not self.host:
            raise JadeError(JR_EINVAL, "not a host buffer")
        raw = (ctypes.c_uint8 * self.nbytes).from_address(self.ptr)
        return np.frombuffer(raw, dtype=NP_DTYPE[self.dtype])


@dataclass
class Kernel:
    runtime: "Runtime"
    handle: int
    spec: dict
    info: dict = field(default_factory=dict)

    def release(self) -> None:
        if self.handle:
            lib().jr_kernel_release(self.handle)
            self.handle = 0


@dataclass
class Execution:
    """src/runtime/mod.rs:23-30 plus per-job device times."""
    host_ms: float
    gpu_ms: float | None
    dispatches: int
    repeats: int
    job_ms: list | None = None


class _Dispatch(ctypes.Structure):
    _fields_ = [("kernel", ctypes.c_void_p), ("buffers", ctypes.POINTER(ctypes.c_void_p)), ("buffer_count", ctypes.c_size_t)]


class Runtime:
    """One device context: a stream, timing events, owned buffers and kernels."""

    def __init__(self, device: int = 0):
        L = lib()
        if L.jr_version() != 1 or L.jr2_version() != 2:
            raise JadeError(JR_EINVAL, "unsupported native runtime ABI")
        e = _err()
        h = ctypes.c_void_p()
        _check(L.jr_create(device, ctypes.byref(h), e, len(e)), e)
        self.ctx = h.value
        self.device = device
        out = ctypes.create_string_buffer(2048)
        _check(L.jr_info(self.ctx, out, len(out), e, len(e)), e)
        self.device_info = out.value.decode()
        self._kernels: list[Kernel] = []

    # -- lifetime
    def close(self) -> None:
        if self.ctx:
            for k in self._kernels:
                k.release()
            lib().jr_destroy(self.ctx)
            self.ctx = None

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def info(self) -> dict:
        """src/runtime/mod.rs:15-21 RuntimeInfo."""
        return {"backend": "CUDA sm_100a built-in kernels", "device": self.device_info,
                "execution": "ordered launches on one persistent non-blocking stream; optional CUDA-graph replay",
                "limitations": ["synchronous API at the public boundary",
                                "FP32, TF32, BF16 and FP16 buffers only"]}

    # -- memory
    def alloc(self, elements: int, dtype: str = "fp32") -> Buffer:
        if elements <= 0:
            raise JadeError(JR_EINVAL, "buffer allocation must be nonempty")
        return self.alloc_bytes(elements * DTYPE_SIZE[dtype], dtype)

    def alloc_bytes(self, nbytes: int, dtype: str = "u8") -> Buffer:
        e = _err()
        p = ctypes.c_void_p()
        _check(lib().jr_alloc(self.ctx, nbytes, ctypes.byref(p), e, len(e)), e)
        return Buffer(self, p.value, nbytes, dtype)

    def host_alloc(self, elements: int, dtype: str = "fp32") -> Buffer:
        e = _err()
        p = ctypes.c_void_p()
        nbytes = elements * DTYPE_SIZE[dtype]
        _check(lib().jr_host_alloc(self.ctx, nbytes, ctypes.byref(p), e, len(e)), e)
        return Buffer(self, p.value, nbytes, dtype, host=True)

    def _own(self, buf: Buffer) -> None:
        if buf.runtime is not self:
            raise JadeError(JR_EINVAL, "buffer belongs to another runtime/device context")
        if buf.freed:
            raise JadeError(JR_EINVAL, "buffer was freed")

    def upload(self, buf: Buffer, data) -> None:
        """Exact transfer: element count must match the buffer (corex.rs:389-411)."""
        self._own(buf)
        arr = np.ascontiguousarray(data, dtype=NP_DTYPE[buf.dtype]).ravel()
        if arr.size != buf.elements:
            raise JadeError(JR_EINVAL, "upload element count must match buffer exactly")
        e = _err()
        _check(lib().jr_upload(self.ctx, buf.ptr, arr.ctypes.data, buf.nbytes, e, len(e)), e)

    def download(self, buf: Buffer, start: int = 0, count: int | None = None) -> np.ndarray:
        """Elements [start, start+count) of a buffer (all of it by default)."""
        self._own(buf)
        count = buf.elements - start if count is None else count
        if start < 0 or count < 1 or start + count > buf.elements:
            raise ValueError(f"range [{start}, {start + count}) outside a buffer of {buf.elements} elements")
        out = np.empty(count, dtype=NP_DTYPE[buf.dtype])
        size = out.itemsize
        e = _err()
        _check(lib().jr_download(self.ctx, buf.ptr + start * size, out.ctypes.data, count * size, e, len(e)), e)
        return out

    def download_f32(self, buf: Buffer, start: int = 0, count: int | None = None) -> np.ndarray:
        out = self.download(buf, start, count)
        if buf.dtype == "bf16":
            return bf16_to_f32(out)
        return out.astype(np.float32)

    # -- kernels
    def compile(self, spec) -> Kernel:
        e = _err()
        h = ctypes.c_void_p()
        text = _spec_text(spec)
        _check(lib().jr_compile(self.ctx, text, ctypes.byref(h), e, len(e)), e)
        out = ctypes.create_string_buffer(1 << 16)
        lib().jr_kernel_info(h.value, out, len(out), e, len(e))
        k = Kernel(self, h.value, json.loads(text), json.loads(out.value or b"{}"))
        self._kernels.append(k)
        return k

    def execute(self, jobs: Iterable, repeats: int = 1, graph: bool = False, per_job: bool = False,
                streams: bool = False) -> Execution:
        """Ordered batch (corex.rs:544-612): every job is validated before any is
        launched; the sequence is replayed ``repeats`` times; returns host and
        device times. ``jobs`` holds (Kernel, [Buffer, ...]) pairs. ``streams``
        (JR_EXEC_STREAMS) runs transfer jobs on their own streams, ordered only by
        the data dependencies of their bindings."""
        jobs = list(jobs)
        if not jobs or repeats <= 0:
            raise JadeError(JR_EINVAL, "execution requires jobs and positive repeats")
        arrays = []
        disp = (_Dispatch * len(jobs))()
        for i, (kernel, bufs) in enumerate(jobs):
            if kernel.runtime is not self:
                raise JadeError(JR_EINVAL, "kernel belongs to another runtime/device context")
            for b in bufs:
                self._own(b)
            arr = (ctypes.c_void_p * len(bufs))(*[b.ptr for b in bufs])
            arrays.append(arr)
            disp[i].kernel = kernel.handle
            disp[i].buffers = ctypes.cast(arr, ctypes.POINTER(ctypes.c_void_p))
            disp[i].buffer_count = len(bufs)
        e = _err()
        gpu = ctypes.c_double(0)
        jm = (ctypes.c_double * len(jobs))() if per_job else None
        t0 = time.perf_counter()
        flags = (JR_EXEC_GRAPH if graph else 0) | (JR_EXEC_STREAMS if streams else 0)
        rc = lib().jr_execute2(self.ctx, disp, len(jobs), repeats, flags, ctypes.byref(gpu), jm, e, len(e))
        host_ms = (time.perf_counter() - t0) * 1e3
        _check(rc, e)
        return Execution(host_ms, gpu.value if gpu.value > 0 else None, len(jobs) * repeats, repeats,
                         list(jm) if per_job else None)

    # -- conveniences used by tests and benches
    def fill(self, buf: Buffer, dist: str, seed: int, stream: int = 0, lo: float = 0.0, hi: float = 1.0,
             offset: int = 0) -> None:
        """Counter-based synthetic input: uniform [lo, hi) or normal(mean=lo, std=hi).
        ``offset``: the generator index of element 0, so that a buffer can hold a
        slice [offset, offset + len) of a larger generated tensor."""
        spec = {"op": "fill", "len": buf.elements, "dist": dist, "seed": seed, "stream": stream, "lo": lo, "hi": hi,
                "dtype": buf.dtype if buf.dtype != "tf32" else "fp32"}
        if offset:
            spec["offset"] = offset
        k = self.compile(spec)
        self.execute([(k, [buf])])
        k.release()
        self._kernels.remove(k)

    # -- peer memory (collectives over NVLink without NCCL)
    def peer_handle(self, buf: Buffer) -> bytes:
        """The 64-byte CUDA IPC handle of a device buffer, for the other ranks."""
        self._own(buf)
        out = ctypes.create_string_buffer(64)
        e = _err()
        _check(lib().jr_peer_handle(self.ctx, buf.ptr, out, e, len(e)), e)
        return out.raw

    def peer_attach(self, buf: Buffer, handles: Sequence[bytes], rank: int) -> None:
        """Maps every other rank's counterpart of `buf` (handles in rank order)."""
        self._own(buf)
        blob = b"".join(handles)
        e = _err()
        _check(lib().jr_peer_attach(self.ctx, buf.ptr, blob, len(handles), rank, e, len(e)), e)

    # -- collectives
    def comm_init(self, nranks: int, rank: int, unique_id: bytes, timeout_ms: int = 60000) -> None:
        e = _err()
        _check(lib().jr_comm_init(self.ctx, nranks, rank, unique_id, timeout_ms, e, len(e)), e)

    def comm_destroy(self) -> None:
        lib().jr_comm_destroy(self.ctx)


def comm_unique_id() -> bytes:
    e = _err()
    buf = ctypes.create_string_buffer(128)
    _check(lib().jr_comm_unique_id(buf, e, len(e)), e)
    return buf.raw


def comm_init_all(runtimes: Sequence[Runtime], timeout_ms: int = 60000) -> None:
    e = _err()
    arr = (ctypes.c_void_p * len(runtimes))(*[r.ctx for r in runtimes])
    _check(lib().jr_comm_init_all(arr, len(runtimes), timeout_ms, e, len(e)), e)
