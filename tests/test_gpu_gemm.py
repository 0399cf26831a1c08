"""GPU parity of the tcgen05 GEMM (BF16 / FP16 / TF32 inputs, FP32 accumulate).

Oracle: src/validation.rs:35-91 (FP64 dot products over the same rounded inputs,
tolerance 2e-5 + coef * sum|a*b|) restated in oracle/oracle.c. For 16-bit inputs
the oracle consumes the stored 16-bit values widened to FP64, so the only error
left is FP32 accumulation (coef = max(2*K*eps32, 2e-6)); TF32 inputs are read
from FP32 storage and truncated inside the tensor core, covered by the
reference's reduced-precision coefficient 0.0012. 16-bit outputs add their own
rounding (2^-8 relative), checked with workloads.rs:224-243 ``compare``.
"""
import numpy as np
import pytest

import jade_compute_b200 as jc
from oracle import oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def rt():
    r = jc.Runtime(0)
    yield r
    r.close()


def operands(rt, m, n, k, dtype, b_nk, seed, nb=None):
    nb = n if nb is None else nb
    a = rt.alloc(m * k, dtype)
    b = rt.alloc(k * nb, dtype)
    rt.fill(a, "uniform", seed=seed, stream=0, lo=-1.0, hi=1.0)
    rt.fill(b, "uniform", seed=seed, stream=1, lo=-1.0, hi=1.0)
    af, bf = rt.download_f32(a), rt.download_f32(b)
    if b_nk:  # stored [N,K]; the oracle wants [K,N]
        bf_kn = np.ascontiguousarray(bf.reshape(nb, k).T).ravel()
    else:
        bf_kn = bf
    return a, b, af, bf_kn


SHAPES = [(128, 256, 64), (128, 256, 128), (256, 512, 512), (1, 8, 8), (33, 40, 24), (200, 300, 136),
          (129, 257, 1024), (512, 768, 4096), (1024, 1024, 1024)]


@pytest.mark.parametrize("dtype", ["bf16", "fp16", "tf32"])
@pytest.mark.parametrize("b_nk", [False, True], ids=["kn", "nk"])
@pytest.mark.parametrize("mnk", SHAPES, ids=str)
def test_tc_gemm_fp32_out(rt, dtype, b_nk, mnk):
    m, n, k = mnk
    a, b, af, bf = operands(rt, m, n, k, dtype, b_nk, seed=m * 7 + n * 3 + k)
    out = rt.alloc(m * n)
    spec = {"op": "gemm", "m": m, "n": n, "k": k, "tiled": True, "dtype": dtype, "b_layout": "nk" if b_nk else "kn"}
    kern = rt.compile(spec)
    if (k * (4 if dtype == "tf32" else 2)) % 16 == 0 and (b_nk or (n * (4 if dtype == "tf32" else 2)) % 16 == 0):
        assert kern.info["path"] == "tcgen05", kern.info
    rt.execute([(kern, [a, b, out])], repeats=2)
    got = rt.download(out)
    rc, v = O.validation_check(m, n, k, af, bf, got, budget=1 << 14, fp16=(dtype == "tf32"))
    assert rc == 0, (rc, v.first_bad_index, v.max_scaled_error, kern.info["impl"])


# 16-bit outputs leave the epilogue in 64-column chunks of packed pairs: whole
# chunks, a partial last chunk (N % 64 != 0), a ragged row (N % 8 != 0: element
# stores) and ragged M
@pytest.mark.parametrize("dtype", ["bf16", "fp16"])
@pytest.mark.parametrize("m,n,k,b_nk,row_scale", [(384, 512, 640, False, False), (130, 1000, 128, True, False),
                                                 (200, 300, 256, True, False), (257, 264, 64, True, True)])
def test_tc_gemm_16bit_out(rt, dtype, m, n, k, b_nk, row_scale):
    a, b, af, bf = operands(rt, m, n, k, dtype, b_nk, seed=3 + n)
    out = rt.alloc(m * n, dtype)
    spec = {"op": "gemm", "m": m, "n": n, "k": k, "tiled": True, "dtype": dtype, "out_dtype": dtype,
            "b_layout": "nk" if b_nk else "kn"}
    bufs = [a, b]
    if row_scale:
        spec["row_scale"] = True
        sc = rt.alloc(m)
        rt.fill(sc, "uniform", seed=5, stream=4, lo=0.5, hi=2.0)
        bufs.append(sc)
    kern = rt.compile(spec)
    assert kern.info["path"] == "tcgen05", kern.info
    rt.execute([(kern, bufs + [out])])
    exp = O.gemm_reference(m, n, k, af, bf)
    if row_scale:
        exp = (exp.reshape(m, n) * rt.download(sc).astype(np.float64)[:, None]).ravel()
    scale = np.abs(exp).max()
    rc, r = O.compare(rt.download_f32(out), exp, 2e-3 * scale, 2 ** -8)
    assert rc == 0, r.max_abs_error


def test_tc_gemm_row_scale_and_residual(rt):
    m, n, k = 256, 512, 384
    a, b, af, bf = operands(rt, m, n, k, "bf16", True, seed=9)
    scale = rt.alloc(m)
    rt.fill(scale, "uniform", seed=9, stream=4, lo=0.5, hi=2.0)
    res = rt.alloc(m * n)
    rt.fill(res, "normal", seed=9, stream=5, lo=0.0, hi=1.0)
    out = rt.alloc(m * n)
    kern = rt.compile({"op": "gemm", "m": m, "n": n, "k": k, "tiled": True, "dtype": "bf16", "b_layout": "nk",
                       "row_scale": True, "epilogue": "residual"})
    rt.execute([(kern, [a, b, scale, res, out])])
    exp = O.gemm_reference(m, n, k, af, bf).reshape(m, n) * rt.download(scale).astype(np.float64)[:, None] \
        + rt.download(res).astype(np.float64).reshape(m, n)
    rc, r = O.compare(rt.download(out), exp.ravel(), 1e-4, 1e-4)
    assert rc == 0, r.max_abs_error


@pytest.mark.parametrize("out_dtype", ["fp32", "bf16"])
def test_tc_gemm_swiglu_epilogue(rt, out_dtype):
    # gate/up weights interleaved in blocks of 128 rows: [g0..g127, u0..u127, g128.., ...]
    m, n, k = 200, 384, 256
    a, b, af, bf_kn = operands(rt, m, n, k, "bf16", True, seed=21, nb=2 * n)
    inv = rt.alloc(m)
    rt.fill(inv, "uniform", seed=21, stream=3, lo=0.5, hi=1.5)
    out = rt.alloc(m * n, out_dtype)
    kern = rt.compile({"op": "gemm", "m": m, "n": n, "k": k, "tiled": True, "dtype": "bf16", "b_layout": "nk",
                       "epilogue": "swiglu", "row_scale": True, "out_dtype": out_dtype})
    assert kern.info["path"] == "tcgen05"
    rt.execute([(kern, [a, b, inv, out])])
    W = bf_kn.reshape(k, 2 * n)  # [K, 2N] with interleaved column blocks
    cols = np.arange(2 * n).reshape(-1, 2, 128)
    gate_cols, up_cols = cols[:, 0, :].ravel(), cols[:, 1, :].ravel()
    A = af.reshape(m, k).astype(np.float64) * rt.download(inv).astype(np.float64)[:, None]
    g = A @ W[:, gate_cols].astype(np.float64)
    u = A @ W[:, up_cols].astype(np.float64)
    h = g / (1 + np.exp(-g)) * u
    tol = (1e-4, 1e-4) if out_dtype == "fp32" else (2e-3 * np.abs(h).max(), 2 ** -8)
    rc, r = O.compare(rt.download_f32(out), h.ravel(), *tol)
    assert rc == 0, r.max_abs_error


def test_tc_gemm_is_deterministic_and_leaves_inputs(rt):
    m, n, k = 512, 512, 512
    a, b, af, bf = operands(rt, m, n, k, "bf16", False, seed=4)
    out1, out2 = rt.alloc(m * n), rt.alloc(m * n)
    kern = rt.compile({"op": "gemm", "m": m, "n": n, "k": k, "tiled": True, "dtype": "bf16"})
    rt.execute([(kern, [a, b, out1]), (kern, [a, b, out2])], repeats=3, graph=True)
    assert np.array_equal(rt.download(out1), rt.download(out2))
    assert np.array_equal(rt.download_f32(a), af)


def test_unaligned_shapes_take_simt_path(rt):
    m, n, k = 31, 47, 19  # K*2 bytes is not a multiple of 16: TMA cannot describe it
    a, b, af, bf = operands(rt, m, n, k, "bf16", False, seed=5)
    out = rt.alloc(m * n)
    kern = rt.compile({"op": "gemm", "m": m, "n": n, "k": k, "tiled": True, "dtype": "bf16"})
    assert kern.info["path"] == "simt"
    rt.execute([(kern, [a, b, out])])
    rc, v = O.validation_check(m, n, k, af, bf, rt.download(out))
    assert rc == 0


# BASELINE configs 5 (square BF16 and TF32 GEMMs up to 16384^3) at full size:
# several 128x256 tiles per persistent CTA, so both TMEM accumulators alternate,
# the [K,N] and [N,K] B layouts, FP32 and BF16 outputs, and the TF32 [K,N]
# transpose path. Checked on validation.rs:35-91's evenly spaced sample (16384
# elements). 16-bit inputs: FP32 accumulation only, coef = 2*K*eps32; a BF16
# output adds its rounding (<= 2^-8 |out| <= 2^-8 sum|a*b|) to the coefficient.
# TF32 inputs: the reference's reduced-precision coefficient 0.0012.
BIG = [("bf16", False, "fp32", 2048), ("bf16", True, "fp32", 2048), ("bf16", False, "bf16", 2048),
       ("bf16", True, "bf16", 2048), ("bf16", False, "fp32", 8192), ("bf16", False, "bf16", 8192),
       ("bf16", True, "fp32", 8192), ("bf16", True, "bf16", 8192), ("bf16", False, "fp32", 16384),
       ("tf32", False, "fp32", 2048), ("tf32", False, "fp32", 4096), ("tf32", True, "fp32", 4096),
       ("tf32", False, "fp32", 8192), ("fp16", False, "fp32", 8192), ("fp16", True, "fp16", 4096)]


@pytest.mark.parametrize("dtype,b_nk,out_dtype,size", BIG, ids=lambda v: str(v))
def test_tc_gemm_baseline_sizes_sampled(rt, dtype, b_nk, out_dtype, size):
    m = n = k = size
    a, b, af, bf = operands(rt, m, n, k, dtype, b_nk, seed=size + (7 if b_nk else 0))
    out = rt.alloc(m * n, out_dtype)
    kern = rt.compile({"op": "gemm", "m": m, "n": n, "k": k, "tiled": True, "dtype": dtype,
                       "b_layout": "nk" if b_nk else "kn", "out_dtype": out_dtype})
    assert kern.info["path"] == "tcgen05", kern.info
    rt.execute([(kern, [a, b, out])], repeats=2)
    got = rt.download_f32(out)
    if dtype == "tf32":
        coef = 0.0012
    else:
        coef = 2 * k * 2.0 ** -23 + {"bf16": 2.0 ** -8, "fp16": 2.0 ** -11}.get(out_dtype, 0.0)
    rc, v = O.validation_check(m, n, k, af, bf, got, budget=1 << 14, coef=coef)
    assert rc == 0, (rc, v.first_bad_index, v.max_scaled_error, kern.info["impl"])
    print(f"{kern.info['impl']} {size}^3: max |err|/sum|a*b| = {v.max_magnitude_error:.2e}, "
          f"max err/tolerance = {v.max_scaled_error:.3f}")
    for x in (a, b, out):
        x.free()


# Split-K: GEMMs with few output tiles and a long K cut K into ranges; each
# (tile, range) writes an FP32 partial and a second kernel sums the partials in
# range order and rounds once. Forced to 4 ranges here (JADE_GEMM_SPLIT_K) so the
# mechanics are covered on short K too. Shapes: several tiles (1024^3), one ragged
# tile with a partial last K block, a tall-K column strip, a single output row.
@pytest.mark.parametrize("dtype,out_dtype", [("bf16", "bf16"), ("bf16", "fp32"), ("fp16", "fp16"), ("tf32", "fp32")])
@pytest.mark.parametrize("m,n,k,b_nk", [(1024, 1024, 1024, False), (100, 200, 1000, True), (256, 136, 4096, True),
                                        (1, 8, 2048, False)], ids=str)
def test_tc_gemm_split_k(rt, monkeypatch, dtype, out_dtype, m, n, k, b_nk):
    a, b, af, bf = operands(rt, m, n, k, dtype, b_nk, seed=k + n)
    out = rt.alloc(m * n, out_dtype)
    monkeypatch.setenv("JADE_GEMM_SPLIT_K", "4")
    kern = rt.compile({"op": "gemm", "m": m, "n": n, "k": k, "tiled": True, "dtype": dtype, "out_dtype": out_dtype,
                       "b_layout": "nk" if b_nk else "kn"})
    assert kern.info["path"] == "tcgen05" and "_splitk4" in kern.info["impl"], kern.info
    rt.execute([(kern, [a, b, out])], repeats=2)
    if out_dtype == "fp32":
        rc, v = O.validation_check(m, n, k, af, bf, rt.download(out), budget=1 << 14, fp16=(dtype == "tf32"))
        assert rc == 0, (rc, v.first_bad_index, v.max_scaled_error, kern.info["impl"])
    else:
        exp = O.gemm_reference(m, n, k, af, bf)
        rc, r = O.compare(rt.download_f32(out), exp, 2e-3 * np.abs(exp).max(), 2 ** -8)
        assert rc == 0, r.max_abs_error


def test_tc_gemm_split_k_deterministic_and_matches_unsplit(rt, monkeypatch):
    m, n, k = 512, 512, 4096  # 8 tiles, 64 K-blocks: the default choice splits
    a, b, af, bf = operands(rt, m, n, k, "bf16", False, seed=12)
    spec = {"op": "gemm", "m": m, "n": n, "k": k, "tiled": True, "dtype": "bf16"}
    split = rt.compile(spec)
    assert rt.compile(dict(spec, k=2048)).info["impl"].find("_splitk") < 0  # 32 K-blocks: too short to split
    monkeypatch.setenv("JADE_GEMM_SPLIT_K", "1")
    whole = rt.compile(spec)
    assert "_splitk" in split.info["impl"] and "_splitk" not in whole.info["impl"]
    o1, o2, o3 = rt.alloc(m * n), rt.alloc(m * n), rt.alloc(m * n)
    rt.execute([(split, [a, b, o1]), (split, [a, b, o2]), (whole, [a, b, o3])], repeats=2)
    assert np.array_equal(rt.download(o1), rt.download(o2))
    # the two summation orders differ only by FP32 rounding
    np.testing.assert_allclose(rt.download(o1), rt.download(o3), rtol=0, atol=1e-3)
