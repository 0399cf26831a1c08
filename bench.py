#!/usr/bin/env python
"""Benchmark of the hot path: causal attention TFLOP/s on BASELINE config 2
(B=4, H=16, S=2048, D=128, BF16 N(0,1), O in BF16), through the C ABI.

Contract (one JSON line on rank 0):
  value      device-timed throughput of the attention kernel, inputs resident in
             HBM, L2 flushed (256 MiB write) between steps; max over ranks.
  e2e        the same metric through the public API with host buffers: each step
             copies Q, K, V from pinned host memory, runs attention and copies O
             back, all as jobs of one batch with the transfers on their own
             streams ordered by data dependencies (JR_EXEC_STREAMS: a step's O
             read-back overlaps the next step's uploads), event-timed.
  roofline   tensor-bound: algorithmic FLOPs per launch / mean launch time vs the
             measured dense BF16 peak; traffic from the committed ncu summary.
  cpu_baseline  the FP64 oracle (the reference's CPU attention restated,
             metal_lab.rs:33-73) on a bounded sample of rows, all host threads.
  components every other BASELINE configuration, each with its roofline and
             the SM clocks of its own timed region: the row kernels and the
             lowered IR expression (config 3); non-causal attention (config 2);
             causal attention B=8 H=32 D=128 at S=4096/8192/16384 split by
             batch x head over the ranks (config 5, strong scaling: a fixed
             problem); the FP32 FFMA GEMM 512^3 (config 1); GEMM 8192^3 BF16 and
             the BF16/TF32 square GEMMs 1024^3..16384^3 split by output columns
             (config 5); the residual MLP block (config 4, tensor parallel with
             one NCCL all-reduce).
  max_err    correctness evidence of this run, taken outside the timed regions
             on rank 0: sampled rows of the headline attention and of the MLP
             block against the FP64 oracle (max |err| / m, m the magnitude of
             the rounded sums: sum_j p_j |v_j| and sum_p |h_p Wd_pc| + |x_c|).
Multi-GPU: one process per GPU (torchrun); each rank runs its own batch x head
shard of the headline attention (weak scaling, no collective on the data path).

--impl reference times the reference's CPU implementation of the path (the
oracle port) on the host cores instead and prints the same metric.
"""
import argparse
import json
import os
import statistics
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "GEMM & causal-attention TFLOP/s, MLP-block tokens/s at 1/2/4/8 B200"
MLP_CHUNKS, MLP_SM_LIMIT = [0], [132]  # tensor-parallel MLP: row blocks (0 = by GPU count), GEMM CTAs
# tensor-parallel MLP collective: nccl all-reduce, peer (NVLink scatter/reduce) or
# auto = peer at 2 and 4 GPUs (measured faster there), nccl otherwise
MLP_COMM = ["auto"]
B, H, S, D = 4, 16, 2048, 128


def headline_config(world):
    """The headline workload as both arms print it: this
    repository's kernels and the reference arm (--impl reference) time the same
    configuration."""
    return {"workload": f"causal attention B={B} H={H} S={S} D={D} BF16, O BF16 (BASELINE configs[1])",
            "global_batch": B * world, "seq_len": S, "heads": H, "head_dim": D,
            "parallelism": f"batch x head shards over {world} GPU(s), no collective",
            "l2": "flushed between steps (256 MiB write)", "flops_per_step_per_gpu": causal_flops(B, H, S, D)}


def causal_flops(b, h, s, d):
    # exact kept (query, key) pairs: s(s+1)/2 per head; QK^T and PV are 2*d each
    return 2.0 * b * h * s * (s + 1) * d


def full_flops(b, h, s, d):
    return 4.0 * b * h * s * s * d


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return {"hbm_gbs": p.get("hbm_gbs", 6650.0), "bf16": p.get("bf16_tflops", 1590.0),
                "bf16_sustained": p.get("bf16_tflops_sustained", 1400.0), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16": 1590.0, "bf16_sustained": 1400.0, "source": "fallback"}


def load_traffic(kernel_key):
    path = os.path.join(ROOT, "profiles", "traffic.json")
    if not os.path.exists(path):
        return None
    with open(path) as f:
        return json.load(f).get(kernel_key)


class ClockSampler:
    """Samples SM clocks and throttle reasons through NVML while the timed region runs."""

    REASONS = {0x8: "hw_slowdown", 0x40: "hw_thermal_slowdown", 0x20: "sw_thermal_slowdown", 0x4: "sw_power_cap",
               0x80: "hw_power_brake_slowdown", 0x1: "gpu_idle", 0x2: "applications_clocks_setting"}

    def __init__(self, device):
        self.samples, self.reasons, self.stop = [], set(), threading.Event()
        self.max_mhz = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(device)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self.nv = None

    def _run(self):
        while not self.stop.is_set():
            try:
                self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
                mask = self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                for bit, name in self.REASONS.items():
                    if mask & bit and name != "gpu_idle":
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(0.01)

    def __enter__(self):
        if self.nv:
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        return self

    def __exit__(self, *a):
        if self.nv:
            self.stop.set()
            self.t.join()

    def summary(self):
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None, "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


def dist_setup():
    from jade_compute_b200 import parallel
    rank, world, local = parallel.env_ranks()
    return parallel.init_process_group(timeout_s=300), world, rank, local


def reduce_max(dist, x):
    from jade_compute_b200 import parallel
    return parallel.max_over_ranks(dist, x)


def barrier(dist):
    if dist is not None:
        dist.barrier()


# ----------------------------------------------------------------------------- CPU
def cpu_attention_sample(seconds, threads, seed=0):
    """Times the FP64 oracle attention (causal, C2 shape) on a sample of rows sized
    to about `seconds`; returns (TFLOP/s, description, threads)."""
    from oracle import oracle as O
    rng = np.random.default_rng(seed)
    n = S * D
    q = rng.standard_normal(n).astype(np.float32)
    k = rng.standard_normal(n).astype(np.float32)
    v = rng.standard_normal(n).astype(np.float32)
    q, k, v = (O.round_bf16(x) for x in (q, k, v))

    def run(rows):
        bh = np.zeros(len(rows), np.int64)
        t0 = time.perf_counter()
        O.attention_rows(S, D, True, q, k, v, bh, rows, threads=threads)
        dt = time.perf_counter() - t0
        return sum(4.0 * D * (int(r) + 1) for r in rows) / dt, dt

    probe = rng.integers(0, S, 8 * threads)
    rate, dt = run(probe)
    per_row = dt / len(probe)
    count = max(threads, int(seconds / max(per_row, 1e-9)))
    rows = rng.integers(0, S, count)
    rate, dt = run(rows)
    return rate / 1e12, f"{count} random causal rows of one head (S={S}, D={D}), FP64 materialized, {dt:.1f} s", threads


def host_threads():
    """Host cores this process may run on. Not the OpenMP default: torchrun sets
    OMP_NUM_THREADS=1 in every rank, and the CPU baselines pass this count
    explicitly to the oracle."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def run_reference(args):
    if int(os.environ.get("RANK", "0")) != 0:
        return 0  # under torchrun only rank 0 times the host implementation
    threads = host_threads()
    per_step = max(1.0, min(10.0, 60.0 / max(args.steps + args.warmup, 1)))
    for _ in range(args.warmup):
        cpu_attention_sample(per_step / 4, threads, seed=1)
    rates, descs, t0 = [], [], time.perf_counter()
    for i in range(args.steps):
        r, desc, _ = cpu_attention_sample(per_step, threads, seed=2 + i)
        rates.append(r)
        descs.append(desc)
    wall = time.perf_counter() - t0
    value = statistics.median(rates)
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": wall * 1e3 / max(args.steps, 1),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f64", "data": "synthetic",
            "config": headline_config(args.gpus),
            "host_work": "FP64 oracle port of the reference's attention (materialized causal rows) on host threads",
            "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": threads, "kind": "port", "sample": descs[0]},
            "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    emit_line(line)
    return 0


# ----------------------------------------------------------------------------- GPU
def attention_bench(rt, jc, steps, warmup, causal, batch):
    n = batch * H * S * D
    q, k, v, o = (rt.alloc(n, "bf16") for _ in range(4))
    for i, buf in enumerate((q, k, v)):
        rt.fill(buf, "normal", seed=1234, stream=i + 10 * (rt.device + 1), lo=0.0, hi=1.0)
    flush_buf = rt.alloc_bytes(256 << 20)
    flush = rt.compile({"op": "l2_flush", "bytes": 256 << 20})
    attn = rt.compile({"op": "attention_online", "heads": H, "seq": S, "dim": D, "causal": causal, "dtype": "bf16",
                       "batch": batch})
    jobs = [(flush, [flush_buf]), (attn, [q, k, v, o])]
    rt.execute(jobs, repeats=max(warmup, 3))
    return jobs, attn, (q, k, v, o), flush_buf


def tensor_roofline(achieved_per_gpu, peaks, which):
    """Tensor-bound roofline of one GPU's share against the measured BF16 peak
    ("bf16" = burst, for a kernel timed alone; "bf16_sustained" inside a long step)."""
    return {"bound": "tensor", "achieved": achieved_per_gpu, "peak": peaks[which], "unit": "TFLOP/s",
            "frac": achieved_per_gpu / peaks[which],
            "peak_source": peaks["source"] + (" burst bf16" if which == "bf16" else " sustained bf16")}


def gemm_bench(rt, dist, world, steps, warmup, peaks, device=0, m=8192):
    """One m^3 BF16 GEMM split by output columns over the ranks (strong scaling):
    rank r computes C[:, cols_r] = A . B[:, cols_r] with B stored [N, K] per shard."""
    from jade_compute_b200 import parallel
    rank = dist.get_rank() if dist is not None else 0
    cols = parallel.split_range(m, world, rank)
    n = len(cols)
    a, b, c = rt.alloc(m * m, "bf16"), rt.alloc(n * m, "bf16"), rt.alloc(m * n, "bf16")
    rt.fill(a, "uniform", seed=5, stream=0, lo=-1, hi=1)
    rt.fill(b, "uniform", seed=5, stream=1 + rank, lo=-1, hi=1)
    layout = "kn" if world == 1 else "nk"
    g = rt.compile({"op": "gemm", "m": m, "n": n, "k": m, "tiled": True, "dtype": "bf16", "out_dtype": "bf16",
                    "b_layout": layout})
    rt.execute([(g, [a, b, c])], repeats=max(warmup, 3))
    clk = ClockSampler(device)  # NVML set-up before the barrier: ranks start the timed region together
    barrier(dist)
    with clk:
        t = rt.execute([(g, [a, b, c])], repeats=steps, per_job=True)
    ms = reduce_max(dist, t.job_ms[0] / steps)
    tflops = 2.0 * m ** 3 / (ms * 1e-3) / 1e12
    for x in (a, b, c):
        x.free()
    return {"workload": f"GEMM {m}^3 BF16 in, FP32 accumulate, BF16 out (BASELINE configs[4]), N-column shards",
            "value": tflops, "unit": "TFLOP/s", "ms_per_step": ms, "n_gpus": world, "scaling": "strong",
            "impl": g.info.get("impl"), "roofline": tensor_roofline(tflops / world, peaks, "bf16"),
            "clocks": clk.summary()}


def row_benches(rt, steps, warmup, peaks, device=0):
    """RMSNorm and softmax on 16384 x 8192 (FP32 and BF16,
    RMSNorm eps 1e-6, weight U[0.5,1.5], softmax logits N(0,1)*4), and the IR
    expression max(2.5x+y, 0) over 2^28 FP32 elements. HBM-bound: algorithmic
    bytes = one read of the input(s) + one write of the output (+ the weight)."""
    R, C, n_expr = 16384, 8192, 1 << 28
    out = []
    flush_buf = rt.alloc_bytes(256 << 20)
    flush = rt.compile({"op": "l2_flush", "bytes": 256 << 20})
    for dtype in ("fp32", "bf16"):
        sz = 4 if dtype == "fp32" else 2
        x, y, w = rt.alloc(R * C, dtype), rt.alloc(R * C, dtype), rt.alloc(C, dtype)
        rt.fill(x, "normal", seed=9, stream=0, lo=0.0, hi=4.0)
        rt.fill(w, "uniform", seed=9, stream=1, lo=0.5, hi=1.5)
        for op, spec, bufs, nbytes in (
                ("rms_norm", {"op": "rms_norm", "rows": R, "cols": C, "epsilon": 1e-6, "dtype": dtype}, [x, w, y],
                 2 * R * C * sz + C * sz),
                ("softmax", {"op": "softmax", "rows": R, "cols": C, "dtype": dtype}, [x, y], 2 * R * C * sz)):
            k = rt.compile(spec)
            jobs = [(flush, [flush_buf]), (k, bufs)]
            rt.execute(jobs, repeats=max(warmup, 3))
            with ClockSampler(device) as clk:
                t = rt.execute(jobs, repeats=steps, per_job=True)
            ms = t.job_ms[1] / steps
            gbs = nbytes / (ms * 1e-3) / 1e9
            out.append({"workload": f"{op} {R}x{C} {dtype} (BASELINE configs[2])", "value": gbs, "unit": "GB/s",
                        "ms_per_step": ms, "roofline": {"bound": "hbm", "achieved": gbs, "peak": peaks["hbm_gbs"],
                                                        "unit": "GB/s", "frac": gbs / peaks["hbm_gbs"]},
                        "impl": k.info.get("impl"), "clocks": clk.summary()})
        for b in (x, y, w):
            b.free()
    a, b, c = rt.alloc(n_expr), rt.alloc(n_expr), rt.alloc(n_expr)
    rt.fill(a, "uniform", seed=10, stream=0, lo=-1, hi=1)
    rt.fill(b, "uniform", seed=10, stream=1, lo=-1, hi=1)
    expr = {"kind": "maximum", "left": {"kind": "add", "left": {"kind": "multiply", "left": {"kind": "input", "binding": 0},
                                                               "right": {"kind": "constant", "value": 2.5}},
                                        "right": {"kind": "input", "binding": 1}},
            "right": {"kind": "constant", "value": 0.0}}
    k = rt.compile({"op": "elementwise", "len": n_expr, "inputs": 2, "expression": expr})
    jobs = [(flush, [flush_buf]), (k, [a, b, c])]
    rt.execute(jobs, repeats=max(warmup, 3))
    with ClockSampler(device) as clk:
        t = rt.execute(jobs, repeats=steps, per_job=True)
    ms = t.job_ms[1] / steps
    gbs = 3 * 4 * n_expr / (ms * 1e-3) / 1e9
    out.append({"workload": "elementwise max(2.5x+y,0) over 2^28 fp32 (BASELINE configs[2])", "value": gbs, "unit": "GB/s",
                "ms_per_step": ms, "roofline": {"bound": "hbm", "achieved": gbs, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                                                "frac": gbs / peaks["hbm_gbs"]}, "impl": k.info.get("impl"), "clocks": clk.summary()})
    for x in (a, b, c, flush_buf):
        x.free()
    return out


def mlp_comm(world):
    """The MLP collective for `world` ranks (--mlp-comm; auto = peer at 2 and 4)."""
    if world <= 1:
        return "nccl"
    if MLP_COMM[0] == "auto":
        return "peer" if world in (2, 4) else "nccl"
    return MLP_COMM[0]


def mlp_bench(rt, dist, world, steps, warmup, peaks, check=False):
    """T=8192, d=4096, ffn=14336 residual MLP, tensor parallel
    over the ranks; the partial outputs are summed by an NCCL all-reduce or by the
    NVLink peer scatter/reduce fused into the down projection (mlp_comm)."""
    from jade_compute_b200 import parallel
    from jade_compute_b200.mlp import ResidualMLP
    from jade_compute_b200.runtime import JadeError
    T, d, ffn = 8192, 4096, 14336
    rank = dist.get_rank() if dist is not None else 0
    if world > 1:
        # NCCL carries the all-reduce in "nccl" mode and, in both modes, the start
        # gate of the timed region below
        parallel.init_comm(rt, dist, timeout_ms=120000)
    # tensor parallel: optionally in row blocks (--mlp-chunks), each block's
    # all-reduce on the collective stream beside the next block's GEMMs, whose grids
    # leave SMs for NCCL. Smaller blocks cost GEMM wave efficiency: one block measured
    # faster than four at 2 GPUs (7.0 vs 6.3 M tokens/s) and than two at 4 GPUs
    # (11.1 vs 9.8), so the default is one block
    comm = mlp_comm(world)

    def build(comm):
        if comm == "peer":
            # the down GEMM scatters its partial rows to their owners over NVLink,
            # owners reduce and push their rows to every rank (csrc/peer.cu)
            chunks, sm_limit = 1, 0
        else:
            chunks = MLP_CHUNKS[0] if MLP_CHUNKS[0] > 0 else 1
            sm_limit = MLP_SM_LIMIT[0] if chunks > 1 else 0
        mlp = ResidualMLP(rt, T, d, ffn, tp=world, rank=rank, chunks=chunks, sm_limit=sm_limit, comm=comm)
        if comm == "peer":
            try:
                mlp.attach(dist)  # raises on every rank if any rank cannot map the peers' buffers
            except JadeError:
                mlp.release()
                raise
        mlp.fill_synthetic(seed=11)
        return mlp, chunks, sm_limit

    fallback = None
    try:
        mlp, chunks, sm_limit = build(comm)
        failure = None
    except JadeError as e:
        mlp, failure = None, e
    if comm == "peer":
        # the peer path's warm-up also decides: a rank whose step fails (a bounded
        # wait that expired) makes every rank fall back to NCCL together
        if mlp is not None:
            try:
                rt.execute(mlp.jobs(), repeats=max(warmup, 3))
            except JadeError as e:
                failure = e
        if not parallel.all_true(dist, failure is None):
            fallback = str(failure or "another rank failed")[:200]
            if mlp is not None:
                mlp.release()
            comm = "nccl"
            mlp, chunks, sm_limit = build(comm)
    elif failure is not None:
        raise failure
    jobs = mlp.jobs()
    lanes = chunks > 1
    rt.execute(jobs, repeats=max(warmup, 3), streams=lanes)
    clk = ClockSampler(rt.device)  # NVML set-up before the barrier: ranks start the timed region together
    gate = None
    if world > 1 and not lanes:
        # the ranks' steps are coupled through the collective, so a rank whose host
        # leaves the CPU barrier first would count the others' lateness (milliseconds
        # of host skew) as its own step time. A one-element NCCL all-reduce ahead of
        # the steps releases every GPU within microseconds; its own time is measured
        # and left out of the region
        gate_buf = rt.alloc(64, "fp32")
        gate = rt.compile({"op": "all_reduce", "len": 64, "dtype": "fp32"})
        rt.execute([(gate, [gate_buf])])
    barrier(dist)
    with clk:
        if gate is not None:
            t = rt.execute([(gate, [gate_buf])] + jobs * steps, per_job=True)
            gate_ms = t.job_ms[0]
            region = t.gpu_ms - gate_ms
            job_ms = [sum(t.job_ms[1 + i::len(jobs)]) for i in range(len(jobs))]
        else:
            t = rt.execute(jobs, repeats=steps, per_job=True, streams=lanes)
            region, job_ms, gate_ms = t.gpu_ms, t.job_ms, None
    job_ms = [x / steps for x in job_ms]
    ms = reduce_max(dist, region / steps)
    flops = 6.0 * T * d * ffn
    per_gpu_tflops = flops / world / (ms * 1e-3) / 1e12
    out = {"workload": f"residual MLP block T={T} d={d} ffn={ffn} BF16 (BASELINE configs[3]), tensor parallel x{world}",
           "value": T / (ms * 1e-3), "unit": "tokens/s", "ms_per_step": ms, "n_gpus": world, "scaling": "strong",
           "tflops": flops / (ms * 1e-3) / 1e12, "job_ms": job_ms,
           "row_blocks": chunks, "gemm_sm_limit": sm_limit or None, "collective": comm if world > 1 else None,
           "collective_fallback": fallback,
           "roofline": {"bound": "tensor", "achieved": per_gpu_tflops, "peak": peaks["bf16_sustained"], "unit": "TFLOP/s",
                        "frac": per_gpu_tflops / peaks["bf16_sustained"], "peak_source": peaks["source"] + " sustained bf16"},
           "kernels": [k.info.get("impl") for k, _ in jobs], "clocks": clk.summary()}
    if world > 1:
        # every rank's region and per-job times (the slowest rank sets ms_per_step)
        import torch
        mine = torch.tensor([region / steps] + job_ms, dtype=torch.float64)
        every = [torch.zeros_like(mine) for _ in range(world)]
        dist.all_gather(every, mine)
        out["per_rank_ms"] = [[round(v, 4) for v in e.tolist()] for e in every]
        out["start_gate_ms"] = gate_ms
        # time of the collective jobs per block (all row blocks), and for the NCCL
        # all-reduce its bus bandwidth: 2 (N-1)/N x bytes / time
        if comm == "nccl":
            coll_ms = sum(ms_ for (k, _), ms_ in zip(jobs, job_ms) if k is mlp.k_ar)
            out["collective_ms"] = coll_ms
            out["allreduce_busbw_gbs"] = 2 * (world - 1) / world * T * d * 2 / (coll_ms * 1e-3) / 1e9 if coll_ms else None
        else:
            out["collective_ms"] = sum(ms_ for (k, _), ms_ in zip(jobs, job_ms) if k in (mlp.k_reduce, mlp.k_gather))
    if check:
        out["max_err"] = mlp_error(rt, mlp, world, seed=11)
    if gate is not None:
        gate.release()
        gate_buf.free()
    if world > 1:
        rt.comm_destroy()
    return out


def c5_attention(rt, dist, world, rank, steps, warmup, peaks, device=0, seqs=(4096, 8192, 16384), causal=True):
    """BASELINE config 5 attention: B=8, H=32, D=128, BF16, S in {4k, 8k, 16k},
    one fixed problem split by batch x head over the ranks (B*H/world heads per
    rank: strong scaling). Value = FLOPs of the whole problem / the slowest rank's
    mean launch time."""
    from jade_compute_b200 import parallel
    out = []
    Bs, Hs = 8, 32
    for seq in seqs:
        heads = parallel.split_range(Bs * Hs, world, rank)
        nh = len(heads)
        n = nh * seq * D
        q, k, v, o = (rt.alloc(n, "bf16") for _ in range(4))
        for i, buf in enumerate((q, k, v)):
            rt.fill(buf, "normal", seed=8, stream=i + 4 * rank, lo=0.0, hi=1.0)
        attn = rt.compile({"op": "attention_online", "heads": nh, "seq": seq, "dim": D, "causal": causal, "dtype": "bf16"})
        rt.execute([(attn, [q, k, v, o])], repeats=max(warmup, 2))
        reps = max(3, min(steps, 20))
        clk = ClockSampler(device)  # NVML set-up before the barrier: ranks start the timed region together
        barrier(dist)
        with clk:
            t = rt.execute([(attn, [q, k, v, o])], repeats=reps, per_job=True)
        ms = reduce_max(dist, t.job_ms[0] / reps)
        flops = causal_flops(Bs, Hs, seq, D) if causal else full_flops(Bs, Hs, seq, D)
        tf = flops / (ms * 1e-3) / 1e12
        out.append({"workload": f"{'causal' if causal else 'non-causal'} attention B={Bs} H={Hs} S={seq} D={D} BF16 "
                                f"(BASELINE configs[4]), batch x head split x{world}",
                    "value": tf, "unit": "TFLOP/s", "ms_per_step": ms, "n_gpus": world, "scaling": "strong",
                    "roofline": tensor_roofline(tf / world, peaks, "bf16"), "impl": attn.info.get("impl"),
                    "clocks": clk.summary()})
        for x in (q, k, v, o):
            x.free()
    return out


def c5_gemms(rt, dist, world, rank, steps, warmup, peaks, device=0, sizes=(1024, 2048, 4096, 8192, 16384)):
    """BASELINE config 5 GEMMs: BF16 and TF32 square M=N=K, inputs U[-1,1], FP32
    out, B and C split by output columns over the ranks (strong scaling)."""
    from jade_compute_b200 import parallel
    out = []
    for dtype in ("bf16", "tf32"):
        for m in sizes:
            cols = parallel.split_range(m, world, rank)
            n = len(cols)
            a, b, c = rt.alloc(m * m, dtype), rt.alloc(n * m, dtype), rt.alloc(m * n, "fp32")
            rt.fill(a, "uniform", seed=7, stream=0, lo=-1, hi=1)
            rt.fill(b, "uniform", seed=7, stream=1 + rank, lo=-1, hi=1)
            g = rt.compile({"op": "gemm", "m": m, "n": n, "k": m, "tiled": True, "dtype": dtype, "b_layout": "nk"})
            reps = max(3, min(steps, int(2e13 / (2.0 * m ** 3)) + 1))
            rt.execute([(g, [a, b, c])], repeats=max(warmup, 2))
            clk = ClockSampler(device)  # NVML set-up before the barrier: ranks start the timed region together
            barrier(dist)
            with clk:
                t = rt.execute([(g, [a, b, c])], repeats=reps, per_job=True)
            ms = reduce_max(dist, t.job_ms[0] / reps)
            tf = 2.0 * m ** 3 / (ms * 1e-3) / 1e12
            out.append({"workload": f"GEMM {m}^3 {dtype} (FP32 out, BASELINE configs[4]), N-split x{world}",
                        "value": tf, "unit": "TFLOP/s", "ms_per_step": ms, "n_gpus": world, "scaling": "strong",
                        "roofline": tensor_roofline(tf / world, peaks, "bf16"), "impl": g.info.get("impl"),
                        "clocks": clk.summary()})
            for x in (a, b, c):
                x.free()
    return out


def sweep(rt, dist, world, rank, steps, warmup, peaks, device=0):
    """BASELINE config 5 on this box: attention first (after the long
    power-capped GEMMs the SM clock recovers slowly), then the GEMMs."""
    return (c5_attention(rt, dist, world, rank, steps, warmup, peaks, device)
            + c5_gemms(rt, dist, world, rank, steps, warmup, peaks, device))


def ffma_bench(rt, steps, warmup, device=0):
    """FP32 GEMM 512^3, A and B ~ U[-1,1] from seed 0, FP32
    FFMA accumulation in k order (bit-exact to the sequential FP32 sum), L2
    flushed between launches. Roofline: the FP32 FFMA peak, SMs x 128 lanes x 2
    FLOP x the maximum SM clock (nominal: no measured FP32 peak exists)."""
    m = 512
    a, b, c = rt.alloc(m * m), rt.alloc(m * m), rt.alloc(m * m)
    rt.fill(a, "uniform", seed=0, stream=0, lo=-1, hi=1)
    rt.fill(b, "uniform", seed=0, stream=1, lo=-1, hi=1)
    flush_buf = rt.alloc_bytes(256 << 20)
    flush = rt.compile({"op": "l2_flush", "bytes": 256 << 20})
    g = rt.compile({"op": "gemm", "m": m, "n": m, "k": m, "tiled": True})
    jobs = [(flush, [flush_buf]), (g, [a, b, c])]
    rt.execute(jobs, repeats=max(warmup, 3))
    reps = max(10, min(steps, 100))
    with ClockSampler(device) as clk:
        t = rt.execute(jobs, repeats=reps, per_job=True)
    ms = t.job_ms[1] / reps
    tf = 2.0 * m ** 3 / (ms * 1e-3) / 1e12
    try:
        import torch
        sms = torch.cuda.get_device_properties(device).multi_processor_count
    except Exception:
        sms = 148
    max_mhz = clk.max_mhz or 1965.0
    peak = sms * 128 * 2 * max_mhz * 1e6 / 1e12
    for x in (a, b, c, flush_buf):
        x.free()
    return {"workload": "FP32 GEMM 512^3 FFMA, k-ordered FP32 accumulation (BASELINE configs[0])", "value": tf,
            "unit": "TFLOP/s", "ms_per_step": ms, "impl": g.info.get("impl"),
            "roofline": {"bound": "ffma", "achieved": tf, "peak": peak, "unit": "TFLOP/s", "frac": tf / peak,
                         "peak_source": f"nominal FP32 FFMA: {sms} SMs x 128 lanes x 2 FLOP x {max_mhz:.0f} MHz"},
            "reference_published_ms": 0.1169, "clocks": clk.summary()}


def attention_error(rt, bufs, batch_heads, causal, seed=0, nrows=48):
    """Max |err| / m of sampled rows of an attention output against the FP64
    oracle (m = sum_j p_j |v_j|), outside any timed region."""
    from oracle import oracle as O
    q, k, v, o = bufs
    rng = np.random.default_rng(seed)
    heads = sorted({0, batch_heads - 1, int(rng.integers(0, batch_heads))})
    fetch = lambda buf: np.concatenate([rt.download_f32(buf, h * S * D, S * D) for h in heads])
    qf, kf, vf, got = (fetch(x) for x in (q, k, v, o))
    bh = rng.integers(0, len(heads), nrows)
    rows = np.concatenate([[0, 1, S - 1], rng.integers(0, S, nrows - 3)])
    ref, mag = O.attention_rows_bound(S, D, causal, qf, kf, vf, bh, rows, threads=host_threads())
    g = got.reshape(len(heads), S, D)[bh, rows]
    ok, scaled, _ = O.bounded_error(g, ref, mag, 2.0 ** -8, 2.0 ** -8 + 1e-4)
    return {"rows": int(nrows), "max_err_over_m": scaled, "within_bound": bool(ok),
            "bound": "|err| <= 2^-8 |ref| + (2^-8 + 1e-4) m"}


def mlp_error(rt, mlp, world, seed, rows=(0, 1, 4097, 8191)):
    """Max |err| / m of sampled rows of the (all-reduced) MLP output against the
    FP64 chain on the BF16 weights of every shard, h rounded to BF16 as stored
    (m = sum_p |h_p Wd_pc| + |x_c|), outside any timed region."""
    from oracle import oracle as O
    from jade_compute_b200.mlp import synthetic_weights
    rows = np.array(rows, np.int64)
    wg, wu, wd = synthetic_weights(rt, mlp.d, mlp.ffn, world, seed)
    x = mlp.download_x()
    ref, mag = O.mlp_rows_bf16h(mlp.d, mlp.ffn, x, np.ones(mlp.d, np.float32), wg, wu, wd, mlp.eps, rows,
                                threads=host_threads())
    got = mlp.download_y_rows(rows)
    err = np.abs(got - ref)
    rms = float(np.sqrt((ref ** 2).mean()))
    return {"rows": len(rows), "max_err_over_m": float((err / mag).max()), "max_err_over_rms": float(err.max() / rms),
            "max_err_over_ref_bf16_ulps": float((err / np.maximum(np.abs(ref), rms * 1e-3)).max() / 2.0 ** -8),
            "tp": world, "collective": mlp.comm if world > 1 else None,
            "partials_dtype": "bf16"}


def kernel_case(rt, case):
    """One kernel family on a small synthetic case (inputs above L2 where the
    kernel is memory-bound), for ncu captures: returns its jobs."""
    def bufs(*specs):
        out = []
        for n, dt in specs:
            b = rt.alloc(n, dt)
            rt.fill(b, "uniform", seed=len(out) + 1, stream=len(out), lo=-1, hi=1)
            out.append(b)
        return out
    if case == "tf32_kn":  # TF32 GEMM with B [K,N]: the transpose pass and the tcgen05 GEMM
        m = 4096
        a, b, c = bufs((m * m, "tf32"), (m * m, "tf32"), (m * m, "fp32"))
        return [(rt.compile({"op": "gemm", "m": m, "n": m, "k": m, "tiled": True, "dtype": "tf32"}), [a, b, c])]
    if case == "gemm_bf16_longk":  # 32 output tiles, K = 8192: split-K (4 ranges) and its reduction
        m, k = 1024, 8192
        a, b, c = bufs((m * k, "bf16"), (k * m, "bf16"), (m * m, "fp32"))
        return [(rt.compile({"op": "gemm", "m": m, "n": m, "k": k, "tiled": True, "dtype": "bf16", "b_layout": "nk"}), [a, b, c])]
    if case in ("ffma512", "ffma2048"):  # FP32 FFMA GEMM (BASELINE configs[0] and a larger square)
        m = 512 if case == "ffma512" else 2048
        a, b, c = bufs((m * m, "fp32"), (m * m, "fp32"), (m * m, "fp32"))
        return [(rt.compile({"op": "gemm", "m": m, "n": m, "k": m, "tiled": True}), [a, b, c])]
    if case in ("swiglu", "axpy", "add"):  # FP32 streaming kernels, 2^26 elements
        n = 1 << 26
        a, b, c = bufs((n, "fp32"), (n, "fp32"), (n, "fp32"))
        spec = {"swiglu": {"op": "swi_glu", "len": n}, "axpy": {"op": "axpy", "len": n, "alpha": 0.5},
                "add": {"op": "add", "len": n}}[case]
        return [(rt.compile(spec), [a, b, c])]
    if case == "swiglu_bf16":
        n = 1 << 27
        a, b, c = bufs((n, "bf16"), (n, "bf16"), (n, "bf16"))
        return [(rt.compile({"op": "swi_glu", "len": n, "dtype": "bf16"}), [a, b, c])]
    if case == "attention_fp32":  # the reference's FP32 online attention (SIMT path), 32 heads x 2048 x 64, causal
        h, s_, d = 32, 2048, 64
        q, k, v, o = bufs(*[(h * s_ * d, "fp32")] * 4)
        return [(rt.compile({"op": "attention_online", "heads": h, "seq": s_, "dim": d, "causal": True}), [q, k, v, o])]
    if case == "mlp_down_k1792":  # the 8-way tensor-parallel shard's down projection with the residual epilogue
        T, d, f = 8192, 4096, 1792
        h, wd, x, y = bufs((T * f, "bf16"), (d * f, "bf16"), (T * d, "bf16"), (T * d, "bf16"))
        return [(rt.compile({"op": "gemm", "m": T, "n": d, "k": f, "tiled": True, "dtype": "bf16", "b_layout": "nk",
                             "out_dtype": "bf16", "epilogue": "residual"}), [h, wd, x, y])]
    if case in ("rms_bf16", "softmax_bf16", "softmax_fp32"):  # BASELINE configs[2] row kernels, 16384 x 8192
        R, C = 16384, 8192
        if case == "rms_bf16":
            x, w, y = bufs((R * C, "bf16"), (C, "bf16"), (R * C, "bf16"))
            return [(rt.compile({"op": "rms_norm", "rows": R, "cols": C, "epsilon": 1e-6, "dtype": "bf16"}), [x, w, y])]
        dt = "fp32" if case == "softmax_fp32" else "bf16"
        x, y = bufs((R * C, dt), (R * C, dt))
        return [(rt.compile({"op": "softmax", "rows": R, "cols": C, "dtype": dt}), [x, y])]
    raise SystemExit(f"unknown kernel case {case}")


KERNEL_CASES = ["tf32_kn", "gemm_bf16_longk", "ffma512", "ffma2048", "swiglu", "axpy", "add", "swiglu_bf16", "attention_fp32", "mlp_down_k1792",
                "rms_bf16", "softmax_bf16", "softmax_fp32"]


def run_only(args):
    """One workload alone (for ncu captures of a single kernel family): prints
    that workload's measurement as the JSON line."""
    dist, world, rank, local = dist_setup()
    import jade_compute_b200 as jc
    peaks = load_peaks()
    rt = jc.Runtime(local)
    try:
        w = args.only
        if w in ("attention", "attention_full"):
            jobs, attn, _, _ = attention_bench(rt, jc, args.steps, args.warmup, w == "attention", B)
            t = rt.execute(jobs, repeats=args.steps, per_job=True)
            ms = t.job_ms[1] / args.steps
            f = causal_flops(B, H, S, D) if w == "attention" else full_flops(B, H, S, D)
            res = {"workload": w, "value": f / (ms * 1e-3) / 1e12, "unit": "TFLOP/s", "ms_per_step": ms, "impl": attn.info.get("impl")}
        elif w == "gemm":
            res = gemm_bench(rt, dist, world, args.steps, args.warmup, peaks, local)
        elif w == "ffma":
            res = ffma_bench(rt, args.steps, args.warmup, local)
        elif w == "mlp":
            res = mlp_bench(rt, dist, world, args.steps, args.warmup, peaks, check=(rank == 0))
        elif w == "rows":
            res = {"workload": "rows", "components": row_benches(rt, args.steps, args.warmup, peaks, local)}
        elif w == "sweep":
            res = {"workload": "sweep", "components": sweep(rt, dist, world, rank, args.steps, args.warmup, peaks, local)}
        elif w in KERNEL_CASES:
            jobs = kernel_case(rt, w)
            t = rt.execute(jobs, repeats=args.steps, per_job=True)
            res = {"workload": w, "impl": [k.info.get("impl") for k, _ in jobs], "ms_per_step": [x / args.steps for x in t.job_ms]}
        else:
            raise SystemExit(f"unknown workload {w}")
        if rank == 0:
            emit_line(res)
    finally:
        rt.close()
    return 0


def run_ours(args):
    if args.only:
        return run_only(args)
    dist, world, rank, local = dist_setup()
    import jade_compute_b200 as jc
    peaks = load_peaks()
    rt = jc.Runtime(local)
    try:
        jobs, attn, (q, k, v, o), flush_buf = attention_bench(rt, jc, args.steps, args.warmup, True, B)
        flops = causal_flops(B, H, S, D)
        clk = ClockSampler(local)  # NVML set-up before the barrier: ranks start the timed region together
        barrier(dist)
        with clk:
            t = rt.execute(jobs, repeats=args.steps, per_job=True)
        attn_ms_total = t.job_ms[1]
        region_ms = t.gpu_ms
        attn_ms_total = reduce_max(dist, attn_ms_total)
        ms_step = attn_ms_total / args.steps
        value = world * flops / (ms_step * 1e-3) / 1e12
        per_gpu = flops / (ms_step * 1e-3) / 1e12
        # end to end through the public API with host buffers
        n = B * H * S * D
        hq, hk, hv, ho = (rt.host_alloc(n, "bf16") for _ in range(4))
        for hb, db in ((hq, q), (hk, k), (hv, v)):
            hb.host_view()[:] = rt.download(db)
        h2d = rt.compile({"op": "copy", "bytes": 2 * n, "direction": "h2d"})
        d2h = rt.compile({"op": "copy", "bytes": 2 * n, "direction": "d2h"})
        e2e_jobs = [(h2d, [hq, q]), (h2d, [hk, k]), (h2d, [hv, v]), (attn, [q, k, v, o]), (d2h, [o, ho])]
        # transfers on their own streams (JR_EXEC_STREAMS), ordered by the data
        # dependencies: a step's O read-back overlaps the next step's uploads
        rt.execute(e2e_jobs, repeats=2, streams=True)
        e2e_steps = max(3, min(args.steps, 50))
        barrier(dist)
        te = rt.execute(e2e_jobs, repeats=e2e_steps, per_job=True, streams=True)
        e2e_ms = reduce_max(dist, te.gpu_ms) / e2e_steps
        e2e_value = world * flops / (e2e_ms * 1e-3) / 1e12
        components = []
        max_err = {"attention_c2": attention_error(rt, (q, k, v, o), B * H, True, seed=rank)}
        if not args.quick:
            # light components first: measured right after the ~1 kW GEMMs and MLP they
            # ran 10-28% slower (partly issue-bound, they follow the SM clock); each
            # records the clocks of its own timed region
            components.extend(row_benches(rt, max(5, min(args.steps, 20)), args.warmup, peaks, local))
            jobs_f, attn_f, bufs_f, fb = attention_bench(rt, jc, args.steps, args.warmup, False, B)
            reps_f = max(5, min(args.steps, 50))
            with ClockSampler(local) as clk_f:
                tf = rt.execute(jobs_f, repeats=reps_f, per_job=True)
            ms_f = tf.job_ms[1] / reps_f
            tf_f = full_flops(B, H, S, D) / (ms_f * 1e-3) / 1e12
            components.append({"workload": f"non-causal attention B={B} H={H} S={S} D={D} BF16 (BASELINE configs[1])",
                               "unit": "TFLOP/s", "value": tf_f, "ms_per_step": ms_f, "impl": attn_f.info.get("impl"),
                               "roofline": tensor_roofline(tf_f, peaks, "bf16"), "clocks": clk_f.summary()})
            for x in (*bufs_f, fb):
                x.free()
            components.extend(c5_attention(rt, dist, world, rank, args.steps, args.warmup, peaks, local))
            components.append(ffma_bench(rt, args.steps, args.warmup, local))
            components.append(gemm_bench(rt, dist, world, max(5, min(args.steps, 20)), args.warmup, peaks, local))
            components.extend(c5_gemms(rt, dist, world, rank, args.steps, args.warmup, peaks, local))
            mlp = mlp_bench(rt, dist, world, max(5, min(args.steps, 20)), args.warmup, peaks, check=(rank == 0))
            if "max_err" in mlp:
                max_err["mlp_c4"] = mlp.pop("max_err")
            components.append(mlp)
        cpu = None
        if rank == 0 and not args.no_cpu:
            from oracle import oracle as O
            thr = host_threads()
            rate, desc, cores = cpu_attention_sample(args.cpu_seconds, thr)
            cpu = {"value": rate, "unit": "TFLOP/s", "cores": cores, "kind": "port", "sample": desc}
        achieved = per_gpu
        traffic = load_traffic("attention_causal_c2")
        line = {
            "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic (counter-based N(0,1), BF16)",
            "config": headline_config(world),
            "kernel": attn.info.get("impl"),
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peaks["bf16"], "unit": "TFLOP/s",
                         "frac": achieved / peaks["bf16"], "peak_source": peaks["source"] + " burst bf16",
                         "traffic": traffic},
            "cpu_baseline": cpu,
            "e2e": {"value": e2e_value, "unit": "TFLOP/s", "h2d_bytes_per_step": 3 * 2 * n, "d2h_bytes_per_step": 2 * n,
                    "ms_per_step": e2e_ms},
            "gpu_launches": 2 * args.steps,
            "clocks": clk.summary(),
            "region_ms": region_ms,
            "components": components,
            "max_err": max_err,
        }
        if rank == 0:
            emit_line(line)
    finally:
        rt.close()
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def main():
    # Native libraries (NCCL's version banner, driver messages) may write to fd 1;
    # route fd 1 to stderr while working so stdout carries exactly one JSON line.
    out_fd = os.dup(1)
    os.dup2(2, 1)
    sys.stdout = os.fdopen(os.dup(2), "w")
    try:
        return _main(out_fd)
    finally:
        sys.stdout.flush()


def emit_line(line):
    os.write(_OUT_FD[0], (json.dumps(line) + "\n").encode())


_OUT_FD = [1]


def _main(out_fd):
    _OUT_FD[0] = out_fd
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--quick", action="store_true", help="headline only, no components")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline sample")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--mlp-chunks", type=int, default=MLP_CHUNKS[0],
                    help="row blocks of the tensor-parallel MLP (0 = one block)")
    ap.add_argument("--mlp-comm", choices=["auto", "nccl", "peer"], default=MLP_COMM[0],
                    help="tensor-parallel MLP collective: NCCL all-reduce, NVLink peer scatter/reduce, or auto "
                         "(peer at 2 and 4 GPUs, NCCL otherwise)")
    ap.add_argument("--mlp-sm-limit", type=int, default=MLP_SM_LIMIT[0],
                    help="persistent CTAs of the tensor-parallel MLP's GEMMs (0 = one per SM)")
    ap.add_argument("--only", choices=["attention", "attention_full", "gemm", "ffma", "mlp", "rows", "sweep"] + KERNEL_CASES,
                    default=None,
                    help="run one workload alone (profiling), printing its own measurement")
    args = ap.parse_args()
    MLP_CHUNKS[0], MLP_SM_LIMIT[0], MLP_COMM[0] = args.mlp_chunks, args.mlp_sm_limit, args.mlp_comm
    if args.warmup < 3:
        args.warmup = 3
    return run_reference(args) if args.impl == "reference" else run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
