"""Residual MLP block on the B200 backend: the reference's six-op synthetic MLP
(src/runtime/workloads.rs:366-525)

    y = x + W_down . ( silu(W_gate . RMSNorm(x)) * (W_up . RMSNorm(x)) )

as four ordered jobs instead of six dispatches:

  1. rms_inv   inv[t] = 1/sqrt(mean(x_t^2) + eps)                (one read of x)
  2. gemm      h = swiglu(diag(inv) . x . Wgu)   tcgen05, B = [gate|up] blocks of
               128 rows interleaved, norm weight folded in (diag(w) W), SwiGLU and
               the row scale applied in the epilogue; h written once in BF16
  3. gemm      y = h . Wd (+ x on rank 0)      tcgen05, residual in the epilogue
  4. all_reduce(y)                              NCCL, only when tensor-parallel

Tensor parallelism over `tp` ranks splits ffn: rank r holds the gate/up columns
and down-projection rows [r*ffn/tp, (r+1)*ffn/tp); the partial outputs are summed
by one all-reduce after the down projection, the residual is added once (rank 0).
With the tokens in row blocks, each block's all-reduce runs on the collective
stream while the next block's GEMMs run (the batch's dependency scheduling
orders them by the buffers they touch).
"""
from __future__ import annotations

import numpy as np

from .runtime import Runtime, f32_to_bf16

BLOCK = 128  # gate/up interleave granularity = half of the GEMM's 256-column tile


def shard_columns(ffn: int, tp: int, rank: int) -> slice:
    if ffn % tp or (ffn // tp) % BLOCK:
        raise ValueError(f"ffn={ffn} must split into {tp} shards that are multiples of {BLOCK}")
    w = ffn // tp
    return slice(rank * w, (rank + 1) * w)


def pack_gate_up(wg: np.ndarray, wu: np.ndarray, norm_weight: np.ndarray) -> np.ndarray:
    """wg, wu: [d, f] (the reference's K x N layout) -> [2f, d] with rows
    [gate block b | up block b] for b = 0..f/128-1, each row scaled by the norm weight."""
    d, f = wg.shape
    g = (wg * norm_weight[:, None]).T  # [f, d]
    u = (wu * norm_weight[:, None]).T
    out = np.empty((2 * f, d), dtype=np.float32)
    for b in range(f // BLOCK):
        out[2 * b * BLOCK:(2 * b + 1) * BLOCK] = g[b * BLOCK:(b + 1) * BLOCK]
        out[(2 * b + 1) * BLOCK:(2 * b + 2) * BLOCK] = u[b * BLOCK:(b + 1) * BLOCK]
    return out


def unpack_gate_up(packed: np.ndarray, d: int):
    """Inverse of pack_gate_up (norm weight left folded in): -> wg, wu as [d, f]."""
    f = packed.shape[0] // 2
    blocks = packed.reshape(f // BLOCK, 2, BLOCK, d)
    return blocks[:, 0].reshape(f, d).T.copy(), blocks[:, 1].reshape(f, d).T.copy()


class ResidualMLP:
    """One tensor-parallel shard of the fused residual MLP, resident on one device.

    ``chunks`` splits the tokens into equal row blocks, each with its own x, inv,
    h and y buffers and its own four jobs; run with ``streams=True`` the
    all-reduce of block c (on the collective stream) overlaps the GEMMs of block
    c+1. ``sm_limit`` caps the persistent CTAs of both GEMMs so that the
    collective's kernels find free SMs beside them."""

    def __init__(self, rt: Runtime, tokens: int, width: int, hidden: int, tp: int = 1, rank: int = 0,
                 eps: float = 1e-5, collective: bool = True, chunks: int = 1, sm_limit: int = 0, comm: str = "nccl"):
        self.rt, self.T, self.d, self.ffn, self.tp, self.rank, self.eps = rt, tokens, width, hidden, tp, rank, eps
        self.f = hidden // tp
        shard_columns(hidden, tp, rank)
        if chunks < 1 or tokens % chunks:
            raise ValueError(f"tokens={tokens} must split into {chunks} equal row blocks")
        if comm not in ("nccl", "peer"):
            raise ValueError("comm must be nccl or peer")
        self.chunks, self.Tc, self.comm = chunks, tokens // chunks, comm
        Tc, d, f = self.Tc, width, self.f
        self.xs = [rt.alloc(Tc * d, "bf16") for _ in range(chunks)]
        self.invs = [rt.alloc(Tc, "fp32") for _ in range(chunks)]
        self.hs = [rt.alloc(Tc * f, "bf16") for _ in range(chunks)]
        self.ys = [rt.alloc(Tc * d, "bf16") for _ in range(chunks)]
        self.wgu = rt.alloc(2 * f * d, "bf16")
        self.wd = rt.alloc(d * f, "bf16")
        base = {"tiled": True, "dtype": "bf16", "b_layout": "nk", "out_dtype": "bf16"}
        if sm_limit:
            base["sm_limit"] = sm_limit
        self.k_inv = rt.compile({"op": "rms_inv", "rows": Tc, "cols": d, "epsilon": eps, "dtype": "bf16"})
        self.k_up = rt.compile({"op": "gemm", "m": Tc, "n": f, "k": d, "epilogue": "swiglu", "row_scale": True, **base})
        down = {"op": "gemm", "m": Tc, "n": d, "k": f, **base}
        self.k_ar = self.k_reduce = self.k_gather = None
        if comm == "peer":
            # the down GEMM stores its partial rows straight into their owners'
            # receive buffers; each owner sums its rows (+ x) and stores them into
            # every rank's y (csrc/peer.cu)
            down.update({"epilogue": "scatter", "ranks": tp, "rank": rank})
            shard = {"rows": Tc, "cols": d, "ranks": tp, "rank": rank, "dtype": "bf16"}
            self.k_reduce = rt.compile({"op": "shard_reduce", "residual": True, **shard})
            self.k_gather = rt.compile({"op": "shard_gather", **shard})
            self.recvs = [rt.alloc(Tc * d, "bf16") for _ in range(chunks)]
            self.flags = rt.alloc_bytes(256)
        else:
            if rank == 0:
                down["epilogue"] = "residual"
            if tp > 1 and collective:
                self.k_ar = rt.compile({"op": "all_reduce", "len": Tc * d, "dtype": "bf16"})
        self.k_down = rt.compile(down)

    def attach(self, dist) -> None:
        """Peer mode: maps the receive buffers, outputs and flags of every rank
        (a collective call: every rank of the block calls it)."""
        from .parallel import share_buffers
        if self.comm != "peer":
            raise ValueError("attach is for comm='peer'")
        share_buffers(self.rt, dist, [*self.recvs, *self.ys, self.flags])

    def release(self) -> None:
        """Frees the block's buffers (detaching peer mappings) and kernels."""
        bufs = [*self.xs, *self.invs, *self.hs, *self.ys, self.wgu, self.wd]
        if self.comm == "peer":
            bufs += [*self.recvs, self.flags]
        for b in bufs:
            b.free()
        for k in (self.k_inv, self.k_up, self.k_down, self.k_ar, self.k_reduce, self.k_gather):
            if k is not None:
                k.release()

    # single-block views (chunks == 1)
    @property
    def x(self):
        if self.chunks != 1:
            raise AttributeError("a chunked block keeps x in row blocks: use xs or download_x()")
        return self.xs[0]

    @property
    def y(self):
        if self.chunks != 1:
            raise AttributeError("a chunked block keeps y in row blocks: use ys or download_y()")
        return self.ys[0]

    def jobs(self):
        j = []
        for c, (x, inv, h, y) in enumerate(zip(self.xs, self.invs, self.hs, self.ys)):
            j += [(self.k_inv, [x, inv]), (self.k_up, [x, self.wgu, inv, h])]
            if self.comm == "peer":
                recv = self.recvs[c]
                j += [(self.k_down, [h, self.wd, recv, self.flags]),
                      (self.k_reduce, [recv, x, y, self.flags]),
                      (self.k_gather, [y, self.flags])]
                continue
            j.append((self.k_down, [h, self.wd, x, y] if self.rank == 0 else [h, self.wd, y]))
            if self.k_ar is not None:
                j.append((self.k_ar, [y]))
        return j

    def flops(self) -> float:
        """Algorithmic FLOPs of this shard: 2*T*d*(2f) + 2*T*f*d."""
        return 6.0 * self.T * self.d * self.f

    # -- host views
    def download_x(self) -> np.ndarray:
        return np.concatenate([self.rt.download_f32(b) for b in self.xs])

    def download_y(self) -> np.ndarray:
        return np.concatenate([self.rt.download_f32(b) for b in self.ys])

    def download_y_rows(self, rows) -> np.ndarray:
        """[len(rows), d] FP32 copies of the listed token rows of y."""
        return np.stack([self.rt.download_f32(self.ys[int(r) // self.Tc], (int(r) % self.Tc) * self.d, self.d) for r in rows])

    # -- weights
    def fill_synthetic(self, seed: int = 0, std: float = 0.02) -> None:
        """BASELINE config 4 inputs: x ~ N(0,1), weights ~ N(0, std), norm weight 1
        (so folding it is the identity); generated on device directly in the packed
        layout, the shard's own stream of the counter-based generator. x is the same
        tensor for any chunking (each block is a slice of one generated stream)."""
        for c, x in enumerate(self.xs):
            self.rt.fill(x, "normal", seed=seed, stream=0, lo=0.0, hi=1.0, offset=c * self.Tc * self.d)
        fill_synthetic_shard(self.rt, self.wgu, self.wd, self.rank, seed, std)

    def load(self, x, norm_weight, wg, wu, wd) -> None:
        """Host FP32 weights in the reference's layout: wg, wu [d, ffn], wd [ffn, d]."""
        cols = shard_columns(self.ffn, self.tp, self.rank)
        xb = f32_to_bf16(np.asarray(x, np.float32).ravel())
        for c, buf in enumerate(self.xs):
            self.rt.upload(buf, xb[c * self.Tc * self.d:(c + 1) * self.Tc * self.d])
        wg = np.asarray(wg, np.float32).reshape(self.d, self.ffn)[:, cols]
        wu = np.asarray(wu, np.float32).reshape(self.d, self.ffn)[:, cols]
        self.rt.upload(self.wgu, f32_to_bf16(pack_gate_up(wg, wu, np.asarray(norm_weight, np.float32)).ravel()))
        wd = np.asarray(wd, np.float32).reshape(self.ffn, self.d)[cols]
        self.rt.upload(self.wd, f32_to_bf16(np.ascontiguousarray(wd.T).ravel()))  # [d, f] = nk layout

def fill_synthetic_shard(rt: Runtime, wgu, wd, rank: int, seed: int = 0, std: float = 0.02) -> None:
    """The packed gate/up weights [2f, d] and down weights [d, f] of shard `rank`
    of the synthetic block (each shard has its own generator streams, so any
    process can regenerate any shard)."""
    rt.fill(wgu, "normal", seed=seed, stream=100 + rank, lo=0.0, hi=std)
    rt.fill(wd, "normal", seed=seed, stream=200 + rank, lo=0.0, hi=std)


def synthetic_weights(rt: Runtime, width: int, hidden: int, tp: int, seed: int = 0, std: float = 0.02):
    """Every shard of the synthetic block's weights regenerated on `rt`'s device
    and returned in the reference's layout as FP32 host arrays: wg, wu [d, ffn]
    and wd [ffn, d] (the values the shards hold, BF16-rounded)."""
    f = hidden // tp
    wg_parts, wu_parts, wd_parts = [], [], []
    wgu, wd = rt.alloc(2 * f * width, "bf16"), rt.alloc(width * f, "bf16")
    try:
        for r in range(tp):
            fill_synthetic_shard(rt, wgu, wd, r, seed, std)
            g, u = unpack_gate_up(rt.download_f32(wgu).reshape(2 * f, width), width)
            wg_parts.append(g)
            wu_parts.append(u)
            wd_parts.append(rt.download_f32(wd).reshape(width, f).T)
    finally:
        wgu.free()
        wd.free()
    return np.concatenate(wg_parts, axis=1), np.concatenate(wu_parts, axis=1), np.concatenate(wd_parts, axis=0)
