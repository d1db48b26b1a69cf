"""The column-block split layer with the exchange over peer memory (CUDA IPC + peer stores
over NVLink) on two GPUs: several consecutive calls (both inbox parities) equal the
one-GPU layer, and a rank that does not publish makes the other rank's call end with a
timeout error after about two seconds instead of hanging (skipped with fewer than two GPUs)."""
import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]
M, K, N = 8, 1024, 3000


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _inputs(call):
    sys.path[:0] = [str(ROOT / "tests")]
    from helpers import int_matrix_m31, random_qm31
    a = int_matrix_m31(M, K, 50 + call)
    b = int_matrix_m31(K, N, 60 + call)
    rng = np.random.default_rng(call)
    return a, b, random_qm31(3 + 12, rng), random_qm31(1, rng)[0]


def _worker(rank, world, port, out_dir):
    sys.path[:0] = [str(ROOT), str(ROOT / "tests"), str(ROOT / "stwo-ml_b200")]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist
    import zkml_b200 as Z
    from zkml_b200.distributed import P2PInbox, column_block, reduce_matmul_layer_colsharded_p2p
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    inbox = P2PInbox(K, ctx=Z.context(rank))
    try:
        lo, hi = column_block(N, rank, world)
        for call in range(3):
            a, b, point, value = _inputs(call)
            blk = torch.from_numpy(np.ascontiguousarray(b[:, lo:hi]).view(np.int32)).cuda()
            ch = Z.PoseidonChannel()
            red, claim = reduce_matmul_layer_colsharded_p2p(Z.GKRClaim(point, value), Z.M31Matrix.from_numpy(a), blk,
                                                            lo, M, K, N, ch, inbox)
            np.savez(os.path.join(out_dir, f"r{rank}_c{call}.npz"), fa=red.final_a_eval, fb=red.final_b_eval,
                     pt=claim.point, dig=np.array([ch.digest() >> (64 * i) & (2**64 - 1) for i in range(4)],
                                                  np.uint64))
        # rank 1 does not publish: rank 0's gather gives up with a timeout
        timed_out = False
        if rank == 0:
            a, b, point, value = _inputs(9)
            blk = torch.from_numpy(np.ascontiguousarray(b[:, lo:hi]).view(np.int32)).cuda()
            try:
                reduce_matmul_layer_colsharded_p2p(Z.GKRClaim(point, value), Z.M31Matrix.from_numpy(a), blk, lo, M,
                                                   K, N, Z.PoseidonChannel(), inbox)
            except Z.ZkmlError as e:
                timed_out = "did not publish" in str(e)
            np.save(os.path.join(out_dir, "timeout.npy"), np.array([timed_out]))
        torch.cuda.synchronize()
        dist.barrier()
    finally:
        inbox.close()
        dist.destroy_process_group()


@pytest.mark.gpu
@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_p2p_split_layer_equals_single_gpu(tmp_path):
    world = 2
    mp.start_processes(_worker, args=(world, _port(), str(tmp_path)), nprocs=world, join=True, start_method="spawn")
    sys.path[:0] = [str(ROOT / "stwo-ml_b200"), str(ROOT / "tests")]
    import zkml_b200 as Z
    for call in range(3):
        a, b, point, value = _inputs(call)
        ch = Z.PoseidonChannel()
        ref, claim = Z.reduce_matmul_layer_with_backend(Z.GKRClaim(point, value), Z.M31Matrix.from_numpy(a),
                                                        Z.M31Matrix.from_numpy(b), M, K, N, ch)
        for r in range(world):
            got = np.load(tmp_path / f"r{r}_c{call}.npz")
            assert (got["fa"] == ref.final_a_eval).all() and (got["fb"] == ref.final_b_eval).all()
            assert (got["pt"] == claim.point).all()
            assert sum(int(got["dig"][i]) << (64 * i) for i in range(4)) == ch.digest()
    assert bool(np.load(tmp_path / "timeout.npy")[0])
