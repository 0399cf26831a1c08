"""Multi-GPU tensor-parallel MLP with the NCCL all-reduce job (2 GPUs, torchrun).

Every rank's all-reduced output must equal the single-GPU unsharded block on the
same inputs within the BF16 MLP tolerance (tests/test_gpu_mlp.py), and all ranks
must hold the same bits."""
import os
import subprocess
import sys

import numpy as np
import pytest

import jade_compute_b200 as jc
from jade_compute_b200.mlp import ResidualMLP
from oracle import oracle as O

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]
HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.mark.skipif(jc.device_count() < 2 if os.path.exists(jc.library_path()) else True, reason="needs 2 GPUs")
@pytest.mark.parametrize("comm", ["nccl", "peer"])
def test_tensor_parallel_mlp_all_reduce_two_gpus(tmp_path, comm):
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", MASTER_ADDR="127.0.0.1")
    port = "29533" if comm == "nccl" else "29534"
    cmd = ["timeout", "-k", "30", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", f"--master-port={port}", os.path.join(HERE, "mp_tp_worker.py"), str(tmp_path), comm]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    y0, y1 = np.load(tmp_path / "y_0.npy"), np.load(tmp_path / "y_1.npy")
    assert np.array_equal(y0, y1)
    rt = jc.Runtime(0)
    try:
        T, d, ffn = 256, 256, 1024
        rng = np.random.default_rng(5)
        x = rng.standard_normal(T * d).astype(np.float32)
        norm = rng.uniform(0.5, 1.5, d).astype(np.float32)
        wg, wu = ((rng.standard_normal((d, ffn)) * 0.05).astype(np.float32) for _ in range(2))
        wd = (rng.standard_normal((ffn, d)) * 0.05).astype(np.float32)
        mlp = ResidualMLP(rt, T, d, ffn)
        mlp.load(x, norm, wg, wu, wd)
        rt.execute(mlp.jobs())
        single = mlp.download_y().astype(np.float64)
    finally:
        rt.close()
    scale = np.sqrt((single ** 2).mean())
    rc, r = O.compare(y0, single, 2e-2 * scale, 2 ** -7)
    assert rc == 0, r.max_abs_error
