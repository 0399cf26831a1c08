"""Worker for tests/test_multigpu.py, launched by torchrun (one process per GPU):
runs the tensor-parallel residual MLP with the NCCL all-reduce job and writes
this rank's all-reduced output to <out_dir>/y_<rank>.npy."""
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import jade_compute_b200 as jc  # noqa: E402
from jade_compute_b200 import parallel  # noqa: E402
from jade_compute_b200.mlp import ResidualMLP  # noqa: E402


def main(out_dir, comm="nccl"):
    rank, world, local = parallel.env_ranks()
    dist = parallel.init_process_group(timeout_s=120)
    rt = jc.Runtime(local)
    parallel.init_comm(rt, dist, timeout_ms=60000)
    T, d, ffn = 256, 256, 1024
    rng = np.random.default_rng(5)
    x = rng.standard_normal(T * d).astype(np.float32)
    norm = rng.uniform(0.5, 1.5, d).astype(np.float32)
    wg, wu = ((rng.standard_normal((d, ffn)) * 0.05).astype(np.float32) for _ in range(2))
    wd = (rng.standard_normal((ffn, d)) * 0.05).astype(np.float32)
    if comm == "peer":
        # partials scattered to their owners over NVLink, reduced and pushed back
        mlp = ResidualMLP(rt, T, d, ffn, tp=world, rank=rank, comm="peer")
        mlp.attach(dist)
        mlp.load(x, norm, wg, wu, wd)
        rt.execute(mlp.jobs(), repeats=3)
    else:
        # two row blocks: block 0's all-reduce runs on the collective stream beside
        # block 1's GEMMs
        mlp = ResidualMLP(rt, T, d, ffn, tp=world, rank=rank, chunks=2, sm_limit=120)
        mlp.load(x, norm, wg, wu, wd)
        rt.execute(mlp.jobs(), repeats=2, streams=True)
    np.save(os.path.join(out_dir, f"y_{rank}.npy"), mlp.download_y())
    dist.barrier()
    rt.comm_destroy()
    rt.close()
    dist.destroy_process_group()


if __name__ == "__main__":
    main(sys.argv[1], *sys.argv[2:])
