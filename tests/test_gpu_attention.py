"""GPU parity of the tcgen05 flash attention (BF16/FP16 inputs, [batch, heads, seq, dim]).

Oracle: the reference's materialized FP64 attention (src/runtime/metal_lab.rs:33-73)
restated in oracle/oracle.c, evaluated on the same 16-bit inputs widened to FP64,
on every row for small cases and on sampled rows at BASELINE sizes.

Tolerance (written here, per output element), derived from where the kernels
round: the softmax weights P are rounded to the input type before P.V (relative
error <= u_in: 2^-8 for BF16, 2^-11 for FP16), so the weighted sum is off by at
most u_in * m with m = sum_j p_j |v_j| (the oracle's magnitude, the attention
analogue of validation.rs:35-91's sum|a*b|); 1e-4 * m more covers FP32
accumulation and the exponential approximations (the FMA-pipe cubic is within
7.5e-5 relative); a 16-bit output adds its own rounding, u_out * |ref|:

    |got - ref| <= u_out * |ref| + (u_in + 1e-4) * m

Each check returns the largest |got - ref| / m it saw; the tests print it so the
achieved error can be read against north_star's 2e-3 (max relative error for
BF16/TF32 inputs with FP32 accumulation).
"""
import numpy as np
import pytest

import jade_compute_b200 as jc
from oracle import oracle as O

pytestmark = pytest.mark.gpu

UNIT_ROUNDOFF = {"bf16": 2.0 ** -8, "fp16": 2.0 ** -11, "fp32": 0.0}
ARITHMETIC = 1e-4


@pytest.fixture(scope="module")
def rt():
    r = jc.Runtime(0)
    yield r
    r.close()


def run_attention(rt, B, H, S, D, causal, dtype="bf16", out_dtype=None, seed=0, heads=None):
    """Runs one attention launch; returns (O rows, Q, K, V) as FP32 arrays for the
    heads listed in `heads` (all when None), in that order."""
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
    heads = list(range(B * H)) if heads is None else list(heads)

    def fetch(buf):
        parts = [rt.download_f32(buf, h * S * D, S * D) for h in heads]
        return np.concatenate(parts).astype(np.float32)

    got, qf, kf, vf = (fetch(x) for x in (o, q, k, v))
    for x in (q, k, v, o):
        x.free()
    return got.reshape(len(heads), S, D), qf, kf, vf


def check(got, qf, kf, vf, S, D, causal, pairs, dtype="bf16", out_dtype=None):
    """pairs: (head index into the fetched heads, row) arrays. Returns the largest
    |got - ref| / m over the checked elements."""
    bh, rows = pairs
    ref, mag = O.attention_rows_bound(S, D, causal, qf, kf, vf, bh, rows, threads=O.max_threads())
    g = got[bh, rows]
    ok, scaled, bad = O.bounded_error(g, ref, mag, UNIT_ROUNDOFF[out_dtype or dtype], UNIT_ROUNDOFF[dtype] + ARITHMETIC)
    assert ok, (bad, g.ravel()[bad], ref.ravel()[bad], mag.ravel()[bad])
    return scaled


@pytest.mark.parametrize("causal", [False, True], ids=["full", "causal"])
@pytest.mark.parametrize("B,H,S,D", [(1, 1, 128, 128), (1, 2, 256, 128), (2, 3, 200, 128), (1, 1, 1, 128),
                                     (1, 2, 129, 64), (1, 1, 384, 64), (2, 2, 1000, 128)])
def test_attention_all_rows(rt, B, H, S, D, causal):
    got, qf, kf, vf = run_attention(rt, B, H, S, D, causal, seed=S + D)
    bh = np.repeat(np.arange(B * H), S)
    rows = np.tile(np.arange(S), B * H)
    print(f"max |err|/m = {check(got, qf, kf, vf, S, D, causal, (bh, rows)):.2e}")


@pytest.mark.parametrize("dtype,out_dtype", [("fp16", None), ("bf16", "fp32"), ("fp16", "fp32")])
def test_attention_dtypes(rt, dtype, out_dtype):
    B, H, S, D = 1, 2, 320, 128
    got, qf, kf, vf = run_attention(rt, B, H, S, D, True, dtype, out_dtype, seed=3)
    bh = np.repeat(np.arange(B * H), S)
    rows = np.tile(np.arange(S), B * H)
    print(f"max |err|/m = {check(got, qf, kf, vf, S, D, True, (bh, rows), dtype, out_dtype):.2e}")


@pytest.mark.parametrize("causal", [False, True], ids=["full", "causal"])
def test_attention_baseline_config2_sampled(rt, causal):
    # B=4, H=16, S=2048, D=128, BF16 N(0,1), O in BF16
    B, H, S, D = 4, 16, 2048, 128
    got, qf, kf, vf = run_attention(rt, B, H, S, D, causal, seed=11)
    rng = np.random.default_rng(0)
    bh = rng.integers(0, B * H, 96)
    rows = np.concatenate([[0, 1, 127, 128, S - 1, S - 128], rng.integers(0, S, 90)])
    print(f"max |err|/m = {check(got, qf, kf, vf, S, D, causal, (bh, rows)):.2e}")


@pytest.mark.parametrize("causal", [False, True], ids=["full", "causal"])
def test_attention_baseline_config2_fp32_out_error(rt, causal):
    # The same workload with an FP32 output, so that only the kernel's own
    # rounding (P in BF16) is measured: the largest |err|/m is north_star's
    # "max relative error" in validation.rs form.
    B, H, S, D = 4, 16, 2048, 128
    got, qf, kf, vf = run_attention(rt, B, H, S, D, causal, out_dtype="fp32", seed=11)
    rng = np.random.default_rng(1)
    bh = rng.integers(0, B * H, 256)
    rows = np.concatenate([np.arange(8), [127, 128, S - 1, S - 128], rng.integers(0, S, 244)])
    scaled = check(got, qf, kf, vf, S, D, causal, (bh, rows), "bf16", "fp32")
    print(f"C2 {'causal' if causal else 'full'} FP32 out: max |err|/m = {scaled:.2e} (P rounding bound 2^-8 = 3.9e-3)")


# BASELINE config 5 attention (B=8, H=32, D=128, BF16) at S = 4096 / 8192 / 16384,
# and non-causal at the same lengths: several persistent rounds of work items per
# SM, head groups sized for L2, the last query and key tiles. Sampled heads are
# fetched alone (each Q/K/V is up to 1 GiB at S=16384).
@pytest.mark.parametrize("S", [4096, 8192, 16384])
@pytest.mark.parametrize("causal", [True, False], ids=["causal", "full"])
def test_attention_baseline_config5_sampled(rt, S, causal):
    B, H, D = 8, 32, 128
    rng = np.random.default_rng(S + causal)
    heads = sorted({0, B * H - 1, *rng.integers(0, B * H, 6).tolist()})
    got, qf, kf, vf = run_attention(rt, B, H, S, D, causal, seed=S // 1024, heads=heads)
    nrow = 192
    bh = rng.integers(0, len(heads), nrow)
    rows = np.concatenate([[0, 1, 127, 128, 255, 256, S - 1, S - 2, S - 128, S - 129], rng.integers(0, S, nrow - 10)])
    scaled = check(got, qf, kf, vf, S, D, causal, (bh, rows))
    print(f"C5 S={S} {'causal' if causal else 'full'}: max |err|/m = {scaled:.2e}")


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
    check(got, qf, kf, vf, S, D, causal, (bh, rows), "bf16", out_dtype)


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
    print(f"max |err|/m = {check(got, qf, kf, vf, S, D, causal, (bh, rows)):.2e}")


@pytest.mark.parametrize("dtype,out_dtype", [("fp16", None), ("bf16", "fp32")])
def test_attention_pair_kernel_dtypes(rt, pair_kernel, dtype, out_dtype):
    B, H, S, D = 1, 1, 2048, 128
    got, qf, kf, vf = run_attention(rt, B, H, S, D, False, dtype, out_dtype, seed=5)
    rows = np.arange(0, S, 3)
    check(got, qf, kf, vf, S, D, False, (np.zeros_like(rows), rows), dtype, out_dtype)


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
    check(got, qf, kf, vf, S, D, False, (np.zeros_like(rows), rows))


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
