"""The product sumcheck split over NCCL ranks on separate GPUs equals the one-GPU proof.

Needs two GPUs (skipped otherwise).  Each rank holds the elements whose index
is its rank modulo the world size and runs its own context on its own GPU; the
per-round exchange is an NCCL all-reduce of 12 words, the final gather an NCCL
all-gather.
"""
import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, n, gather_local, out_dir, mode="python"):
    sys.path[:0] = [str(ROOT), str(ROOT / "tests"), str(ROOT / "stwo-ml_b200")]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist
    from zkml_b200 import PoseidonChannel
    from zkml_b200.distributed import GpuSumcheckSession, prove_product_sharded, shard_of
    from helpers import uniform_m31
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    try:
        a = uniform_m31(n, 21)
        b = uniform_m31(n, 22)
        la = torch.from_numpy(shard_of(a, rank, world).view(np.int32)).cuda()
        lb = torch.from_numpy(shard_of(b, rank, world).view(np.int32)).cuda()
        if mode == "python":
            proof = prove_product_sharded(la, lb, n, PoseidonChannel(), session=GpuSumcheckSession(device=rank),
                                          gather_local=gather_local)
        else:
            from zkml_b200 import context
            from zkml_b200.distributed import ShmExchange, TorchExchange, job_nonce, prove_product_sharded_native
            ex = (ShmExchange(f"zkml_nccl_t_{port}", world, rank, max_gather_bytes=32 * (n // world),
                              nonce=job_nonce()) if mode == "shm"
                  else TorchExchange())
            proof = prove_product_sharded_native(la, lb, n, PoseidonChannel(), ex, gather_local=gather_local,
                                                 ctx=context(rank))
            ex.close()
        np.savez(os.path.join(out_dir, f"r{rank}.npz"), ch=proof.challenges, fa=proof.final_a, fb=proof.final_b,
                 gathered=proof.gathered_at)
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("n,gather_local,mode", [(1 << 20, 1 << 12, "python"), (1 << 16, 1 << 16, "python"),
                                                 (1 << 20, 1 << 12, "shm"), (1 << 20, 1 << 12, "nccl"),
                                                 (1 << 12, 1 << 16, "shm")])
def test_nccl_sharded_equals_single_gpu(n, gather_local, mode, tmp_path):
    world = 2
    mp.start_processes(_worker, args=(world, _port(), n, gather_local, str(tmp_path), mode), nprocs=world, join=True,
                       start_method="spawn")
    sys.path[:0] = [str(ROOT / "stwo-ml_b200"), str(ROOT / "tests")]
    import zkml_b200 as Z
    from helpers import uniform_m31
    a = uniform_m31(n, 21)
    b = uniform_m31(n, 22)
    ref = Z.GpuBackend(0).reduce_matmul_layer(Z.M31Matrix.from_numpy(a.reshape(1, n)),
                                              Z.M31Matrix.from_numpy(b.reshape(n, 1)), [], [], n,
                                              Z.PoseidonChannel())
    for r in range(world):
        got = np.load(tmp_path / f"r{r}.npz")
        np.testing.assert_array_equal(got["ch"], ref.challenges)
        np.testing.assert_array_equal(got["fa"], ref.final_a_eval)
        np.testing.assert_array_equal(got["fb"], ref.final_b_eval)
