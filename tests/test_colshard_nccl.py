"""A matmul layer split by column blocks over two NCCL ranks on separate GPUs equals the
one-GPU layer (skipped with fewer than two GPUs)."""
import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]
M, K, N = 16, 5120, 13824


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, out_dir):
    sys.path[:0] = [str(ROOT), str(ROOT / "tests"), str(ROOT / "stwo-ml_b200")]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist
    import zkml_b200 as Z
    from zkml_b200.distributed import column_block, reduce_matmul_layer_colsharded
    from helpers import int_matrix_m31, random_qm31
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    try:
        a = int_matrix_m31(M, K, 41)
        b = int_matrix_m31(K, N, 42)
        point, value = random_qm31(4 + 14, np.random.default_rng(5)), random_qm31(1, np.random.default_rng(6))[0]
        lo, hi = column_block(N, rank, world)
        blk = torch.from_numpy(np.ascontiguousarray(b[:, lo:hi]).view(np.int32)).cuda()
        ch = Z.PoseidonChannel()
        red, claim = reduce_matmul_layer_colsharded(Z.GKRClaim(point, value), Z.M31Matrix.from_numpy(a), blk, lo,
                                                    M, K, N, ch, ctx=Z.context(rank))
        np.savez(os.path.join(out_dir, f"r{rank}.npz"), fa=red.final_a_eval, fb=red.final_b_eval, pt=claim.point,
                 dig=np.array([ch.digest() >> (64 * i) & (2**64 - 1) for i in range(4)], np.uint64))
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_nccl_column_blocks_equal_single_gpu(tmp_path):
    world = 2
    mp.start_processes(_worker, args=(world, _port(), str(tmp_path)), nprocs=world, join=True, start_method="spawn")
    sys.path[:0] = [str(ROOT / "stwo-ml_b200"), str(ROOT / "tests")]
    import zkml_b200 as Z
    from helpers import int_matrix_m31, random_qm31
    a = int_matrix_m31(M, K, 41)
    b = int_matrix_m31(K, N, 42)
    point, value = random_qm31(4 + 14, np.random.default_rng(5)), random_qm31(1, np.random.default_rng(6))[0]
    ch = Z.PoseidonChannel()
    ref, claim = Z.reduce_matmul_layer_with_backend(Z.GKRClaim(point, value), Z.M31Matrix.from_numpy(a),
                                                    Z.M31Matrix.from_numpy(b), M, K, N, ch)
    dig = ch.digest()
    for r in range(world):
        got = np.load(tmp_path / f"r{r}.npz")
        assert (got["fa"] == ref.final_a_eval).all() and (got["fb"] == ref.final_b_eval).all()
        assert (got["pt"] == claim.point).all()
        assert sum(int(got["dig"][i]) << (64 * i) for i in range(4)) == dig
