"""The sharded product sumcheck over the peer mesh (CUDA IPC + peer stores over NVLink, the
round words added inside the round kernels) on 2 and 4 GPUs: consecutive proofs of several
sizes equal the oracle's single proof bit for bit, the gather of too-short vectors included;
and a rank that stops calling makes the other ranks' next call end with a timeout error after
about two seconds instead of hanging (skipped with fewer GPUs)."""
import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]
CASES = [(1 << 16, 1 << 8), (1 << 12, 2), (1 << 14, 1 << 6), (1 << 6, 1 << 16), (1 << 16, 1 << 8)]


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _vectors(n, case):
    sys.path[:0] = [str(ROOT / "tests")]
    from helpers import uniform_m31
    return uniform_m31(n, 300 + case), uniform_m31(n, 400 + case)


def _worker(rank, world, port, out_dir):
    sys.path[:0] = [str(ROOT), str(ROOT / "tests"), str(ROOT / "stwo-ml_b200")]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist
    import zkml_b200 as Z
    from zkml_b200.distributed import PeerMesh, prove_product_sharded_mesh, shard_of
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    mesh = PeerMesh(ctx=Z.context(rank), max_gather_bytes=32 << 16)
    try:
        for case, (n, gl) in enumerate(CASES):
            a, b = _vectors(n, case)
            la = torch.from_numpy(shard_of(a, rank, world).view(np.int32)).cuda()
            lb = torch.from_numpy(shard_of(b, rank, world).view(np.int32)).cuda()
            ch = Z.PoseidonChannel()
            proof = prove_product_sharded_mesh(la, lb, n, ch, mesh, gather_local=gl)
            rp = np.stack([np.concatenate([p.c0, p.c1, p.c2]) for p in proof.round_polys])
            np.savez(os.path.join(out_dir, f"r{rank}_c{case}.npz"), rp=rp, ch=proof.challenges, fa=proof.final_a,
                     fb=proof.final_b, gathered=proof.gathered_at)
        torch.cuda.synchronize()
        dist.barrier()
        # every rank but 0 stops: rank 0's first split round gives up with a timeout
        if rank == 0:
            a, b = _vectors(1 << 16, 0)
            la = torch.from_numpy(shard_of(a, rank, world).view(np.int32)).cuda()
            lb = torch.from_numpy(shard_of(b, rank, world).view(np.int32)).cuda()
            timed_out = False
            try:
                prove_product_sharded_mesh(la, lb, 1 << 16, Z.PoseidonChannel(), mesh, gather_local=1 << 8)
            except Z.ZkmlError as e:
                timed_out = "did not arrive" in str(e)
            np.save(os.path.join(out_dir, "timeout.npy"), np.array([timed_out]))
        torch.cuda.synchronize()
        dist.barrier()
    finally:
        mesh.close()
        dist.destroy_process_group()


@pytest.mark.gpu
@pytest.mark.parametrize("world", [2, 4])
def test_mesh_sharded_product_equals_oracle(world, tmp_path):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    mp.start_processes(_worker, args=(world, _port(), str(tmp_path)), nprocs=world, join=True, start_method="spawn")
    sys.path[:0] = [str(ROOT / "tests")]
    import oracle_lib
    for case, (n, gl) in enumerate(CASES):
        a, b = _vectors(n, case)
        ref = oracle_lib.reduce_matmul_layer(a.reshape(1, n), b.reshape(n, 1), np.zeros((0, 4), np.uint32),
                                             np.zeros((0, 4), np.uint32), oracle_lib.new_channel(), mode=0,
                                             nthreads=4)
        for r in range(world):
            got = np.load(tmp_path / f"r{r}_c{case}.npz")
            assert (got["rp"] == np.stack(ref["round_polys"])).all(), (case, r)
            assert (got["fa"] == ref["final_a"]).all() and (got["fb"] == ref["final_b"]).all()
    assert bool(np.load(tmp_path / "timeout.npy")[0])
