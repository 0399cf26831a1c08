"""Multi-GPU plumbing: one process per GPU, torch.distributed for the host-side
control plane (rank discovery, barriers, broadcasting the NCCL id, max-over-ranks
timing), this library's NCCL communicator for the data-path collective.

Sharding (the reference has no multi-device code; this follows the scheme of
the build's scope table):
  * attention: the batch*heads index space is split into contiguous ranges,
    no collective;
  * GEMM: B and C are split by output columns (N), A replicated, no collective;
  * MLP: tensor parallel over ffn (see mlp.py), one all-reduce after the down
    projection.
"""
from __future__ import annotations

import datetime
import os
from typing import Callable, Optional

from . import runtime as _rt


def env_ranks():
    """(rank, world, local_rank) from the launcher's environment (torchrun)."""
    return (int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")),
            int(os.environ.get("LOCAL_RANK", "0")))


def init_process_group(timeout_s: float = 120.0):
    """CPU (gloo) process group for control traffic; None when single-process.
    Rendezvous uses MASTER_ADDR/MASTER_PORT (127.0.0.1 on one box)."""
    rank, world, _ = env_ranks()
    if world <= 1:
        return None
    import torch.distributed as dist
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    if not dist.is_initialized():
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=timeout_s))
    return dist


def split_range(total: int, parts: int, index: int) -> range:
    """Contiguous, balanced split of range(total): the first total % parts parts get one extra."""
    if parts < 1 or not 0 <= index < parts:
        raise ValueError("bad split")
    base, extra = divmod(total, parts)
    start = index * base + min(index, extra)
    return range(start, start + base + (1 if index < extra else 0))


def broadcast_bytes(dist, payload: Optional[bytes], src: int = 0, size: int = 128) -> bytes:
    """Broadcast a fixed-size byte string from rank `src` over the CPU group."""
    import torch
    t = torch.zeros(size, dtype=torch.uint8)
    if dist.get_rank() == src:
        if payload is None or len(payload) != size:
            raise ValueError("source rank must provide the payload")
        t[:] = torch.frombuffer(bytearray(payload), dtype=torch.uint8)
    dist.broadcast(t, src=src)
    return bytes(t.tolist())


def max_over_ranks(dist, value: float) -> float:
    if dist is None:
        return value
    import torch
    t = torch.tensor([value], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def init_comm(rt: "_rt.Runtime", dist, timeout_ms: int = 60000,
              make_id: Callable[[], bytes] = _rt.comm_unique_id) -> None:
    """NCCL communicator over every rank of `dist` for this runtime's device."""
    rank, world = dist.get_rank(), dist.get_world_size()
    uid = make_id() if rank == 0 else None
    uid = broadcast_bytes(dist, uid, src=0, size=128)
    rt.comm_init(world, rank, uid, timeout_ms)


def all_gather_bytes(dist, payload: bytes) -> list:
    """Every rank's fixed-size byte string, in rank order, over the CPU group."""
    import torch
    world = dist.get_world_size()
    mine = torch.frombuffer(bytearray(payload), dtype=torch.uint8)
    out = [torch.zeros(len(payload), dtype=torch.uint8) for _ in range(world)]
    dist.all_gather(out, mine)
    return [bytes(t.tolist()) for t in out]


def all_true(dist, flag: bool) -> bool:
    """True when `flag` holds on every rank (a collective over the CPU group)."""
    if dist is None:
        return bool(flag)
    import torch
    t = torch.tensor([1 if flag else 0], dtype=torch.int32)
    dist.all_reduce(t, op=dist.ReduceOp.MIN)
    return bool(t.item())


def share_buffers(rt: "_rt.Runtime", dist, buffers) -> None:
    """Attaches each buffer to its counterparts on every rank (CUDA IPC handles
    exchanged over the CPU group; every rank passes the same sequence of
    same-sized buffers). Single process: attaches with one rank.

    Every rank takes the same collective steps whatever fails: the handles of all
    buffers travel in one exchange with a status byte, each rank maps them
    locally, and the ranks then agree on the outcome; if exporting or mapping
    failed on any rank, every rank raises JadeError (buffers mapped so far stay
    attached until they are freed)."""
    rank = dist.get_rank() if dist is not None else 0
    buffers = list(buffers)
    failure = None
    try:
        mine = b"".join(rt.peer_handle(b) for b in buffers)
    except _rt.JadeError as e:
        mine, failure = b"\0" * (64 * len(buffers)), e
    payload = bytes([failure is None]) + mine
    every = all_gather_bytes(dist, payload) if dist is not None else [payload]
    if failure is None and not all(p[0] for p in every):
        failure = _rt.JadeError(_rt.JR_EINVAL, "a rank could not export its peer handles")
    if failure is None:
        try:
            for i, buf in enumerate(buffers):
                rt.peer_attach(buf, [p[1 + 64 * i:1 + 64 * (i + 1)] for p in every], rank)
        except _rt.JadeError as e:
            failure = e
    if not all_true(dist, failure is None):
        raise failure or _rt.JadeError(_rt.JR_EINVAL, "another rank could not attach its peer buffers")
