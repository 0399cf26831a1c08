"""Failure detection on the GPU without a fault: every wait in the tcgen05
kernels is bounded and, on expiry, records a code in the context's mapped error
word; the batch then returns JR_ETIMEOUT and the context stays usable. The
wait_probe op runs one such bounded wait on an mbarrier that nothing arrives on,
with a short limit, so this path is exercised deliberately: no trap, no device
assert, no bad address, no unbounded loop."""
import numpy as np
import pytest

import jade_compute_b200 as jc
from jade_compute_b200.runtime import JadeError
from oracle import oracle as O

pytestmark = pytest.mark.gpu
JR_ETIMEOUT = 4


def test_expired_device_wait_reports_timeout_and_the_context_recovers():
    rt = jc.Runtime(0)
    try:
        probe = rt.compile({"op": "wait_probe", "limit_ns": 50_000_000})  # 50 ms
        out = rt.alloc(2)
        for attempt in range(2):  # the error word is cleared after each report
            with pytest.raises(JadeError) as e:
                rt.execute([(probe, [out])])
            assert e.value.code == JR_ETIMEOUT, e.value
            assert "bounded wait expired" in e.value.message and "wait probe" in e.value.message
            waited_ns, satisfied = rt.download(out)
            assert satisfied == 0.0 and waited_ns >= 50e6, (attempt, waited_ns)
        # the same context runs ordinary work afterwards, with correct results
        m, n, k = 256, 512, 384
        a, b, c = rt.alloc(m * k, "bf16"), rt.alloc(k * n, "bf16"), rt.alloc(m * n)
        rt.fill(a, "uniform", seed=3, stream=0, lo=-1, hi=1)
        rt.fill(b, "uniform", seed=3, stream=1, lo=-1, hi=1)
        g = rt.compile({"op": "gemm", "m": m, "n": n, "k": k, "tiled": True, "dtype": "bf16"})
        rt.execute([(g, [a, b, c])])
        rc, v = O.validation_check(m, n, k, rt.download_f32(a), rt.download_f32(b), rt.download(c))
        assert rc == 0, v.max_scaled_error
    finally:
        rt.close()


def test_expiry_inside_a_batch_stops_the_batch_report():
    # jobs after the expired wait still run (the stream is not poisoned), and the
    # batch as a whole reports the expiry
    rt = jc.Runtime(0)
    try:
        probe = rt.compile({"op": "wait_probe", "limit_ns": 10_000_000})
        out = rt.alloc(2)
        x = rt.alloc(4096)
        fill = rt.compile({"op": "fill", "len": 4096, "dist": "uniform", "seed": 9, "stream": 0, "lo": 0.0, "hi": 1.0})
        with pytest.raises(JadeError) as e:
            rt.execute([(probe, [out]), (fill, [x])])
        assert e.value.code == JR_ETIMEOUT
        vals = rt.download(x)
        assert np.isfinite(vals).all() and 0.0 <= vals.min() and vals.max() < 1.0
        rt.execute([(fill, [x])])  # and the next batch succeeds
    finally:
        rt.close()


def test_peer_attachment_ends_with_its_buffer():
    # a freed buffer's peer mappings close with it: a new buffer (possibly at the
    # same address) is not attached until it is shared again
    from jade_compute_b200.parallel import share_buffers
    rt = jc.Runtime(0)
    try:
        y, flags = rt.alloc(128 * 8, "bf16"), rt.alloc_bytes(256)
        share_buffers(rt, None, [y, flags])
        gather = rt.compile({"op": "shard_gather", "rows": 128, "cols": 8, "ranks": 1, "rank": 0, "dtype": "bf16"})
        rt.execute([(gather, [y, flags])])
        flags.free()
        fresh = rt.alloc_bytes(256)
        with pytest.raises(JadeError, match="not attached to peer memory"):
            rt.execute([(gather, [y, fresh])])
        share_buffers(rt, None, [fresh])
        rt.execute([(gather, [y, fresh])])
    finally:
        rt.close()
