"""GPU parity of the tcgen05 flash attention (BF16/FP16 inputs, [batch, heads, seq, dim]).

Oracle: the reference's materialized FP64 attention (src/runtime/metal_lab.rs:33-73)
restated in oracle/oracle.c, evaluated on the same 16-bit inputs widened to FP64,
on every row for small cases and on sampled rows at BASELINE sizes.

Tolerance (written here, per element): |got - ref| <= atol + rtol*|ref| with
atol = 4e-3 (P is rounded to the 16-bit input type before P.V, relative error
2^-9 per weight; |V| <= ~5 for N(0,1) inputs) and rtol = 2^-8 for 16-bit outputs
(one output rounding) or 1e-3 for FP32 outputs.
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


def run_attention(rt, B, H, S, D, causal, dtype="bf16", out_dtype=None, seed=0):
    n = B * H * S * D
    q, k, v = (rt.alloc(n, dtype) for _ in range(3))
    for i, buf in enumerate((q, k, v)):
        rt.fill(buf, "normal", seed=seed, stream=i, lo=0.0, hi=1.0)
    spec = {"op": "attention_online", "heads": H, "seq": S, "dim": D, "causal": causal, "dtype": dtype, "batch": B}
    if out_dtype:
        spec["out_dtype"] = out_dtype
    o = rt.alloc(n, out_dtype or dtype)
    kern = rt.compile(spec)
    assert kern.info["path"] == "tcgen05", kern.info
    rt.execute([(kern, [q, k, v, o])], repeats=2)
    qf, kf, vf = (rt.download_f32(x) if dtype == "bf16" else rt.download(x).astype(np.float32) for x in (q, k, v))
    got = rt.download_f32(o) if (out_dtype or dtype) == "bf16" else rt.download(o).astype(np.float32)
    return got.reshape(B * H, S, D), qf, kf, vf


def check(got, qf, kf, vf, S, D, causal, pairs, out16):
    bh, rows = pairs
    ref = O.attention_rows(S, D, causal, qf, kf, vf, bh, rows, threads=O.max_threads())
    g = got[bh, rows]
    rtol = 2 ** -8 if out16 else 1e-3
    rc, r = O.compare(g.ravel(), ref.ravel(), 4e-3, rtol)
    assert rc == 0, (r.first_bad_index, r.max_abs_error)
    return np.abs(g - ref).max()


@pytest.mark.parametrize("causal", [False, True], ids=["full", "causal"])
@pytest.mark.parametrize("B,H,S,D", [(1, 1, 128, 128), (1, 2, 256, 128), (2, 3, 200, 128), (1, 1, 1, 128),
                                     (1, 2, 129, 64), (1, 1, 384, 64), (2, 2, 1000, 128)])
def test_attention_all_rows(rt, B, H, S, D, causal):
    got, qf, kf, vf = run_attention(rt, B, H, S, D, causal, seed=S + D)
    bh = np.repeat(np.arange(B * H), S)
    rows = np.tile(np.arange(S), B * H)
    check(got, qf, kf, vf, S, D, causal, (bh, rows), True)


@pytest.mark.parametrize("dtype,out_dtype", [("fp16", None), ("bf16", "fp32"), ("fp16", "fp32")])
def test_attention_dtypes(rt, dtype, out_dtype):
    B, H, S, D = 1, 2, 320, 128
    got, qf, kf, vf = run_attention(rt, B, H, S, D, True, dtype, out_dtype, seed=3)
    bh = np.repeat(np.arange(B * H), S)
    rows = np.tile(np.arange(S), B * H)
    check(got, qf, kf, vf, S, D, True, (bh, rows), (out_dtype or dtype) != "fp32")


@pytest.mark.parametrize("causal", [False, True], ids=["full", "causal"])
def test_attention_baseline_config2_sampled(rt, causal):
    # B=4, H=16, S=2048, D=128, BF16 N(0,1), O in BF16
    B, H, S, D = 4, 16, 2048, 128
    got, qf, kf, vf = run_attention(rt, B, H, S, D, causal, seed=11)
    rng = np.random.default_rng(0)
    bh = rng.integers(0, B * H, 96)
    rows = np.concatenate([[0, 1, 127, 128, S - 1, S - 128], rng.integers(0, S, 90)])
    check(got, qf, kf, vf, S, D, causal, (bh, rows), True)


@pytest.mark.parametrize("B,H,S,D,causal,out_dtype", [
    (2, 80, 2048, 128, True, None),    # 1280 items in 3 head groups (K/V of 64 heads per L2 group)
    (1, 150, 1100, 128, True, "fp32"),  # 9 q tiles: the heaviest item of every head has one tile
    (3, 50, 1000, 64, False, None),     # head dim 64, 600 equal items
    (1, 300, 4200, 64, True, None),     # 300 heads in 5 groups, tail tile of 104 keys
], ids=["groups", "odd-tiles-fp32", "d64-full", "groups-d64-tail"])
def test_attention_persistent_items(rt, B, H, S, D, causal, out_dtype):
    # the two-tile kernel is persistent: each CTA walks several (head, q-tile pair)
    # items, reusing its Q buffers, TMEM and O staging across them
    got, qf, kf, vf = run_attention(rt, B, H, S, D, causal, out_dtype=out_dtype, seed=S + H)
    rng = np.random.default_rng(S)
    bh = np.concatenate([[0, B * H - 1, B * H // 2], rng.integers(0, B * H, 93)])
    rows = np.concatenate([[0, S - 1, 127, 128 % S], rng.integers(0, S, 92)])
    check(got, qf, kf, vf, S, D, causal, (bh, rows), out_dtype is None)


def test_attention_uniform_rows_kat(rt):
    # metal_lab.rs:471-484 restated: Q = K = 0 gives uniform weights, so each
    # output row is the mean of the visible V rows (exact in any precision order
    # up to the 16-bit rounding of V and of the 1/count factor).
    B, H, S, D = 1, 1, 256, 64
    n = B * H * S * D
    q, k, v, o = rt.alloc(n, "bf16"), rt.alloc(n, "bf16"), rt.alloc(n, "bf16"), rt.alloc(n, "fp32")
    rt.fill(v, "normal", seed=1, lo=0.0, hi=1.0)
    kern = rt.compile({"op": "attention_online", "heads": H, "seq": S, "dim": D, "causal": True, "dtype": "bf16",
                       "out_dtype": "fp32"})
    rt.execute([(kern, [q, k, v, o])])
    V = rt.download_f32(v).reshape(S, D).astype(np.float64)
    exp = np.cumsum(V, axis=0) / np.arange(1, S + 1)[:, None]
    assert np.abs(rt.download(o).reshape(S, D) - exp).max() < 3e-3


# ---------------------------------------------------------------- CTA-pair kernel
# The cta_group::2 kernel (attention_tc2.cu: S triple-buffered in TMEM, two softmax
# warps per lane quarter on alternating key steps, speculative maxima) runs
# non-causal head-dim-128 shapes whose work items fill its 74 CTA pairs better than
# the two-tile kernel's 148 SMs; JADE_ATTENTION_KERNEL=pair forces it, which these
# tests do so that its causal path stays covered too.

def pair_impl(kern):
    return "pair" in kern.info.get("impl", "")


@pytest.fixture
def pair_kernel(monkeypatch):
    monkeypatch.setenv("JADE_ATTENTION_KERNEL", "pair")


def kernel_impl(rt, B, H, S, causal, D=128):
    return rt.compile({"op": "attention_online", "heads": H, "seq": S, "dim": D, "causal": causal, "dtype": "bf16",
                       "batch": B}).info["impl"]


def test_attention_kernel_choice(rt, monkeypatch):
    # measured rule: causal always two-tile; non-causal 512 items (3.46 rounds of the
    # two-tile kernel's 148 SMs) go to the pair kernel, 2048 items do not
    assert "pair" not in kernel_impl(rt, 4, 16, 2048, True)
    assert "pair" in kernel_impl(rt, 4, 16, 2048, False)
    assert "pair" not in kernel_impl(rt, 8, 16, 4096, False)
    assert "pair" not in kernel_impl(rt, 16, 16, 1024, False)
    monkeypatch.setenv("JADE_ATTENTION_KERNEL", "two_tile")
    assert "pair" not in kernel_impl(rt, 4, 16, 2048, False)
    monkeypatch.setenv("JADE_ATTENTION_KERNEL", "pair")
    assert "pair" in kernel_impl(rt, 4, 16, 2048, True)
    with pytest.raises(jc.JadeError, match="head dim 128"):
        kernel_impl(rt, 1, 1, 256, False, D=64)
    monkeypatch.setenv("JADE_ATTENTION_KERNEL", "fastest")
    with pytest.raises(jc.JadeError, match="pair or two_tile"):
        kernel_impl(rt, 1, 1, 256, False)


@pytest.mark.parametrize("B,H,S,causal", [(1, 2, 2048, False), (1, 1, 2100, False), (2, 1, 2304, False),
                                          (1, 1, 6144, True), (1, 1, 6200, True)],
                         ids=["full2048", "full2100tail", "full2304", "causal6144", "causal6200tail"])
def test_attention_pair_kernel(rt, pair_kernel, B, H, S, causal):
    D = 128
    got, qf, kf, vf = run_attention(rt, B, H, S, D, causal, seed=S + 7)
    kern = rt.compile({"op": "attention_online", "heads": H, "seq": S, "dim": D, "causal": causal, "dtype": "bf16", "batch": B})
    assert pair_impl(kern), kern.info
    rng = np.random.default_rng(S)
    nrow = 512 if causal else 1024
    bh = rng.integers(0, B * H, nrow)
    # both CTAs of a pair, tile edges, the last (partial) tile and random rows
    edges = [min(e, S - 1) for e in (0, 1, 127, 128, 255, 256, S - 1, S - 2, (S // 256) * 256, (S // 256) * 256 + 128)]
    rows = np.concatenate([edges, rng.integers(0, S, nrow - len(edges))])
    check(got, qf, kf, vf, S, D, causal, (bh, rows), True)


@pytest.mark.parametrize("dtype,out_dtype", [("fp16", None), ("bf16", "fp32")])
def test_attention_pair_kernel_dtypes(rt, pair_kernel, dtype, out_dtype):
    B, H, S, D = 1, 1, 2048, 128
    got, qf, kf, vf = run_attention(rt, B, H, S, D, False, dtype, out_dtype, seed=5)
    rows = np.arange(0, S, 3)
    check(got, qf, kf, vf, S, D, False, (np.zeros_like(rows), rows), (out_dtype or dtype) != "fp32")


def test_attention_pair_kernel_rescales(rt, pair_kernel):
    # scores that grow along the keys force the running maximum up by far more
    # than 2^8 at every key step: the speculative P is redone and O rescaled each step
    B, H, S, D = 1, 1, 2048, 128
    n = S * D
    key = np.arange(S, dtype=np.float32)[:, None]
    qh = np.ones((S, D), np.float32) * 0.5
    kh = np.repeat(key * (0.04 / 0.5) / 8, D, axis=1).astype(np.float32)
    vh = np.random.default_rng(9).standard_normal((S, D)).astype(np.float32)
    bufs = [rt.alloc(n, "bf16") for _ in range(4)]
    for b, h in zip(bufs[:3], (qh, kh, vh)):
        rt.upload(b, jc.runtime.f32_to_bf16(h.ravel()))
    kern = rt.compile({"op": "attention_online", "heads": H, "seq": S, "dim": D, "causal": False, "dtype": "bf16"})
    assert pair_impl(kern), kern.info
    rt.execute([(kern, bufs)])
    got = rt.download_f32(bufs[3]).reshape(1, S, D)
    qf, kf, vf = (rt.download_f32(b) for b in bufs[:3])
    rows = np.arange(0, S, 7)
    check(got, qf, kf, vf, S, D, False, (np.zeros_like(rows), rows), True)


def test_attention_pair_kernel_uniform_kat(rt, pair_kernel):
    # Q = K = 0: every non-causal output row is the mean of all V rows
    B, H, S, D = 1, 1, 2048, 128
    n = S * D
    q, k, v, o = rt.alloc(n, "bf16"), rt.alloc(n, "bf16"), rt.alloc(n, "bf16"), rt.alloc(n, "fp32")
    rt.fill(v, "normal", seed=2, lo=0.0, hi=1.0)
    kern = rt.compile({"op": "attention_online", "heads": H, "seq": S, "dim": D, "causal": False, "dtype": "bf16",
                       "out_dtype": "fp32"})
    assert pair_impl(kern), kern.info
    rt.execute([(kern, [q, k, v, o])])
    V = rt.download_f32(v).reshape(S, D).astype(np.float64)
    assert np.abs(rt.download(o).reshape(S, D) - V.mean(axis=0)[None]).max() < 2e-3
