"""GPU parity of the residual MLP block (src/runtime/workloads.rs:366-525).

1. The reference's own six-op FP32 MLP (RMSNorm -> gate/up GEMM -> SwiGLU ->
   down GEMM -> add) through the ordered batch, inputs and tolerance exactly as
   workloads.rs:390-481 (xorshift32 inputs, compare at 5e-5/5e-5).
2. The fused BF16 block (rms_inv -> tcgen05 GEMM with row-scale + SwiGLU
   epilogue -> tcgen05 GEMM with residual epilogue), against the FP64 chain
   evaluated on the same effective BF16 weights, with h rounded to BF16 where the
   block stores it (oracle or_mlp_rows_ex). Tolerance, from where the block
   rounds: y is stored in BF16 (2^-8 relative); the rest is the down
   projection's FP32 accumulation over K = ffn terms (tensor-core accumulation,
   plus rare one-ulp differences in the BF16 h), bounded as validation.rs:35-91
   bounds an FP32 sum: coef = 2 * K * eps32 times m = sum_p |h_p * Wd[p][c]| +
   |x_c|. So |got - ref| <= 2^-8 |ref| + 2 K eps32 m. The tests print the largest
   |got - ref| / m.
3. Tensor-parallel sharding math on one GPU: the shards' partial outputs sum to
   the unsharded block (the all-reduce itself is covered by the multi-GPU test);
   each BF16 partial adds its own rounding, 2^-8 |partial|.
"""
import json
import math

import numpy as np
import pytest

import jade_compute_b200 as jc
from jade_compute_b200.mlp import ResidualMLP, unpack_gate_up
from oracle import oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def rt():
    r = jc.Runtime(0)
    yield r
    r.close()


@pytest.mark.parametrize("batch,width,hidden", [(8, 128, 256), (64, 512, 1024), (3, 17, 33)])
def test_reference_six_op_fp32_mlp(rt, batch, width, hidden):
    m, w, h = batch, width, hidden
    x = O.values(m * w, 0x1234, 1.0)
    norm = np.ones(w, np.float32)
    wg = O.values(w * h, 0x3333, 1.0 / math.sqrt(np.float32(w)))
    wu = O.values(w * h, 0x4444, 1.0 / math.sqrt(np.float32(w)))
    wd = O.values(h * w, 0x5555, 1.0 / math.sqrt(np.float32(h)))

    def res(v):
        b = rt.alloc(len(v))
        rt.upload(b, v)
        return b

    xg, ng, wgg, wug, wdg = map(res, (x, norm, wg, wu, wd))
    normalized, gate, up, act, proj, out = (rt.alloc(n) for n in (m * w, m * h, m * h, m * h, m * w, m * w))
    eps = 1e-5
    k = [rt.compile(s) for s in (
        {"op": "rms_norm", "rows": m, "cols": w, "epsilon": eps},
        {"op": "gemm", "m": m, "n": h, "k": w, "tiled": True},
        {"op": "gemm", "m": m, "n": h, "k": w, "tiled": True},
        {"op": "swi_glu", "len": m * h},
        {"op": "gemm", "m": m, "n": w, "k": h, "tiled": True},
        {"op": "add", "len": m * w})]
    jobs = [(k[0], [xg, ng, normalized]), (k[1], [normalized, wgg, gate]), (k[2], [normalized, wug, up]),
            (k[3], [gate, up, act]), (k[4], [act, wdg, proj]), (k[5], [proj, xg, out])]
    rt.execute(jobs, repeats=3)
    expected = O.mlp_rows(w, h, x, norm, wg, wu, wd, float(np.float32(eps)), np.arange(m))
    rc, r = O.compare(rt.download(out), expected.ravel(), 5e-5, 5e-5)
    assert rc == 0, r.max_abs_error
    # batched replay and graph replay give the same bits as a single pass
    first = rt.download(out)
    rt.execute(jobs, repeats=2, graph=True)
    assert np.array_equal(rt.download(out), first)


def effective_oracle(rt, mlp_shards, rows):
    """FP64 chain on the weights the device actually holds (BF16, norm folded),
    h rounded to BF16; returns (reference rows, magnitude m)."""
    d = mlp_shards[0].d
    x = mlp_shards[0].download_x()
    wg_parts, wu_parts, wd_parts = [], [], []
    for s in mlp_shards:
        wg, wu = unpack_gate_up(rt.download_f32(s.wgu).reshape(2 * s.f, d), d)
        wg_parts.append(wg)
        wu_parts.append(wu)
        wd_parts.append(rt.download_f32(s.wd).reshape(d, s.f).T)
    wg = np.concatenate(wg_parts, axis=1)
    wu = np.concatenate(wu_parts, axis=1)
    wd = np.concatenate(wd_parts, axis=0)
    ffn = wg.shape[1]
    return O.mlp_rows_bf16h(d, ffn, x, np.ones(d, np.float32), wg, wu, wd, mlp_shards[0].eps, rows,
                            threads=O.max_threads())


EPS32 = 2.0 ** -23


def check_mlp(got_rows, oracle, ffn, out_rel=2.0 ** -8, extra=None):
    ref, mag = oracle
    coef = 2 * ffn * EPS32
    if extra is not None:  # per-element rounding already in got (summed BF16 partials)
        mag = mag + extra / coef
    ok, scaled, bad = O.bounded_error(got_rows, ref, mag, out_rel, coef)
    assert ok, (bad, got_rows.ravel()[bad], ref.ravel()[bad], mag.ravel()[bad], coef)
    print(f"max |err|/m = {scaled:.2e} (bound {coef:.1e} + output rounding)")
    return scaled


@pytest.mark.parametrize("T,d,ffn", [(256, 256, 512), (200, 384, 1024)])
def test_fused_mlp_small_all_rows(rt, T, d, ffn):
    mlp = ResidualMLP(rt, T, d, ffn, eps=1e-5)
    rng = np.random.default_rng(T + d)
    x = rng.standard_normal(T * d).astype(np.float32)
    norm = rng.uniform(0.5, 1.5, d).astype(np.float32)
    wg = (rng.standard_normal((d, ffn)) * 0.05).astype(np.float32)
    wu = (rng.standard_normal((d, ffn)) * 0.05).astype(np.float32)
    wd = (rng.standard_normal((ffn, d)) * 0.05).astype(np.float32)
    mlp.load(x, norm, wg, wu, wd)
    rt.execute(mlp.jobs(), repeats=2)
    got = mlp.download_y().reshape(T, d)
    rows = np.arange(T)
    check_mlp(got, effective_oracle(rt, [mlp], rows), ffn)


def test_fused_mlp_baseline_config4_sampled(rt):
    # T=8192, d=4096, ffn=14336, BF16 W ~ N(0,0.02), x ~ N(0,1)
    T, d, ffn = 8192, 4096, 14336
    mlp = ResidualMLP(rt, T, d, ffn, eps=1e-5)
    mlp.fill_synthetic(seed=3)
    rt.execute(mlp.jobs(), repeats=1)
    rows = np.array([0, 1, 4095, 8191, 127, 128, 5000, 6001])
    got = mlp.download_y_rows(rows)
    check_mlp(got, effective_oracle(rt, [mlp], rows), ffn)


def test_tensor_parallel_shards_sum_to_block(rt):
    T, d, ffn, tp = 256, 256, 1024, 4
    rng = np.random.default_rng(7)
    x = rng.standard_normal(T * d).astype(np.float32)
    norm = np.ones(d, np.float32)
    wg, wu = ((rng.standard_normal((d, ffn)) * 0.05).astype(np.float32) for _ in range(2))
    wd = (rng.standard_normal((ffn, d)) * 0.05).astype(np.float32)
    shards = [ResidualMLP(rt, T, d, ffn, tp=tp, rank=r, collective=False) for r in range(tp)]
    total = np.zeros(T * d, np.float64)
    partial_size = np.zeros(T * d, np.float64)
    for s in shards:
        s.load(x, norm, wg, wu, wd)
        rt.execute(s.jobs())
        part = s.download_y().astype(np.float64)
        total += part
        partial_size += np.abs(part)
    # each partial is rounded to BF16 once: 2^-8 |partial| per shard, no output rounding
    check_mlp(total.reshape(T, d), effective_oracle(rt, shards, np.arange(T)), ffn, out_rel=0.0,
              extra=(2.0 ** -8 * partial_size).reshape(T, d))


def test_row_blocks_and_collective_lane_give_the_same_bits(rt):
    # the block split into 4 row blocks with capped GEMM grids, run with the
    # dependency-scheduled streams, equals the single block bit for bit (each
    # output row's sums do not depend on the row tiling)
    T, d, ffn = 1024, 512, 1024
    whole = ResidualMLP(rt, T, d, ffn)
    blocks = ResidualMLP(rt, T, d, ffn, chunks=4, sm_limit=100)
    assert all("sm_limit" in k.spec for k in (blocks.k_up, blocks.k_down))
    for m in (whole, blocks):
        m.fill_synthetic(seed=5)
    assert np.array_equal(whole.download_x(), blocks.download_x())
    rt.execute(whole.jobs())
    rt.execute(blocks.jobs(), repeats=2, streams=True)
    assert np.array_equal(whole.download_y(), blocks.download_y())
    rows = np.array([0, 255, 256, 1023])
    assert np.array_equal(blocks.download_y_rows(rows), whole.download_y().reshape(T, d)[rows])


@pytest.mark.parametrize("chunks", [1, 2])
def test_peer_collective_path_on_one_rank(rt, chunks):
    # comm="peer" with one rank: the down GEMM's scatter epilogue, shard_reduce (+x)
    # and shard_gather run their whole data path on one GPU (the arrival flags are
    # this rank's own). The partial is rounded to BF16 before the reduction adds x,
    # one rounding more than the residual epilogue: 2^-8 |partial| more slack.
    T, d, ffn = 1024, 512, 1024
    ref = ResidualMLP(rt, T, d, ffn)
    peer = ResidualMLP(rt, T, d, ffn, comm="peer", chunks=chunks)
    peer.attach(None)
    assert "scatter" in peer.k_down.info["impl"] or "scatter" in json.dumps(peer.k_down.spec)
    for m in (ref, peer):
        m.fill_synthetic(seed=8)
    rt.execute(ref.jobs())
    rt.execute(peer.jobs(), repeats=3)  # arrival numbers advance every repeat
    first = peer.download_y()
    rt.execute(peer.jobs(), repeats=2, graph=True)  # the epochs live on the device: graphs replay too
    assert np.array_equal(peer.download_y(), first)
    rows = np.arange(0, T, 37)
    oracle = effective_oracle(rt, [peer], rows)
    partial = np.abs(oracle[0] - peer.download_x().reshape(T, d)[rows])
    check_mlp(first.reshape(T, d)[rows], oracle, ffn, extra=2.0 ** -8 * partial)
