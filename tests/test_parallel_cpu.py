"""Host-side multi-process logic on CPU (gloo, world_size 2): id broadcast,
max-over-ranks timing, range splitting, tensor-parallel MLP sharding math (the
per-rank partial outputs reduced with an all-reduce equal the unsharded block),
and failure detection without a GPU (a rank that never joins makes the other's
collective fail within its timeout)."""
import os
import socket

import numpy as np
import pytest


def free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, scenario, q):
    os.environ.update({"RANK": str(rank), "WORLD_SIZE": str(world), "LOCAL_RANK": str(rank),
                       "MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port)})
    try:
        import torch
        from jade_compute_b200 import parallel as P
        from jade_compute_b200.mlp import pack_gate_up, shard_columns, unpack_gate_up
        if scenario == "never_join" and rank == 1:
            q.put((rank, "left"))
            return
        if scenario == "never_join":
            try:  # the missing rank is detected at rendezvous or at the first collective
                dist = P.init_process_group(timeout_s=4)
                dist.barrier()
                q.put((rank, "no error"))
            except Exception as e:
                q.put((rank, "detected: " + type(e).__name__))
            return
        dist = P.init_process_group(timeout_s=10 if scenario != "leave_between_steps" else 5)
        if scenario.startswith("share"):
            # peer-buffer sharing agrees on failure: a rank that cannot export (or
            # map) its handles makes every rank raise, with no collective left waiting
            from jade_compute_b200.runtime import JadeError

            class FakeRuntime:
                def __init__(self):
                    self.attached = []

                def peer_handle(self, buf):
                    if scenario == "share_export_fails" and rank == 1:
                        raise JadeError(1, "export refused")
                    return bytes([rank, buf]) + b"\0" * 62

                def peer_attach(self, buf, handles, r):
                    if scenario == "share_attach_fails" and rank == 0:
                        raise JadeError(2, "map refused")
                    assert [h[:2] for h in handles] == [bytes([q, buf]) for q in range(world)] and r == rank
                    self.attached.append(buf)

            rt = FakeRuntime()
            try:
                P.share_buffers(rt, dist, [7, 8, 9])
                result = "attached " + ",".join(map(str, rt.attached))
            except JadeError as e:
                result = "raised " + e.message
            dist.barrier()  # both ranks are still in step: no collective was left waiting
            dist.destroy_process_group()
            q.put((rank, result))
            return
        if scenario == "leave_between_steps":
            dist.barrier()  # step 1 completes on both ranks
            if rank == 1:
                q.put((rank, "left"))
                q.close()
                q.join_thread()  # flush the message before leaving
                os._exit(0)  # leaves between steps, with nothing in flight
            try:
                import datetime
                # step 2: the peer is gone; the monitored barrier names it within its timeout
                dist.monitored_barrier(timeout=datetime.timedelta(seconds=5))
                q.put((rank, "no error"))
            except Exception as e:
                q.put((rank, "detected: " + type(e).__name__))
            return
        if scenario == "basic":
            uid = P.broadcast_bytes(dist, bytes(range(128)) if rank == 0 else None)
            assert uid == bytes(range(128))
            assert P.max_over_ranks(dist, float(rank + 1)) == float(world)
            parts = [P.split_range(10, world, r) for r in range(world)]
            assert sum(len(p) for p in parts) == 10 and parts[0].start == 0 and parts[-1].stop == 10
            # tensor-parallel MLP: the sum of per-rank partials equals the full block
            rng = np.random.default_rng(0)
            T, d, ffn = 8, 16, 512
            x = rng.standard_normal((T, d))
            wg, wu = rng.standard_normal((d, ffn)) * 0.1, rng.standard_normal((d, ffn)) * 0.1
            wd = rng.standard_normal((ffn, d)) * 0.1
            norm = rng.uniform(0.5, 1.5, d)
            xn = x / np.sqrt((x * x).mean(1, keepdims=True) + 1e-5)

            def block(wg_, wu_, wd_):
                g, u = (xn * norm) @ wg_, (xn * norm) @ wu_
                return (g / (1 + np.exp(-g)) * u) @ wd_

            cols = shard_columns(ffn, world, rank)
            packed = pack_gate_up(wg[:, cols].astype(np.float32), wu[:, cols].astype(np.float32),
                                  np.ones(d, np.float32))
            g2, u2 = unpack_gate_up(packed, d)
            assert np.array_equal(g2, wg[:, cols].astype(np.float32))
            part = block(wg[:, cols], wu[:, cols], wd[cols]) + (x if rank == 0 else 0)
            t = torch.from_numpy(part.copy())
            dist.all_reduce(t)
            full = block(wg, wu, wd) + x
            assert np.allclose(t.numpy(), full, atol=1e-10)
            dist.barrier()
            dist.destroy_process_group()
            q.put((rank, "ok"))
    except Exception as e:  # pragma: no cover - reported to the parent
        q.put((rank, f"error: {e!r}"))


def _run(scenario, world=2, timeout=120):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, scenario, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    for _ in range(world):
        r, msg = q.get(timeout=timeout)
        out[r] = msg
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    return out


def test_gloo_two_ranks_control_plane_and_tp_math():
    out = _run("basic")
    assert out == {0: "ok", 1: "ok"}, out


def test_rank_that_never_joins_is_detected_on_host():
    out = _run("never_join")
    assert out[1] == "left"
    assert out[0].startswith("detected"), out


def test_rank_that_leaves_between_steps_is_detected_on_host():
    out = _run("leave_between_steps")
    assert out[1] == "left"
    assert out[0].startswith("detected"), out


def test_peer_buffer_sharing_attaches_every_buffer():
    assert _run("share_ok") == {0: "attached 7,8,9", 1: "attached 7,8,9"}


@pytest.mark.parametrize("scenario", ["share_export_fails", "share_attach_fails"])
def test_peer_buffer_sharing_fails_on_every_rank_together(scenario):
    out = _run(scenario)
    assert all(v.startswith("raised") for v in out.values()), out
    failing = 1 if scenario == "share_export_fails" else 0
    assert "refused" in out[failing], out
