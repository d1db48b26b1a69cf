"""The GKR chain prover with the weight openings' Merkle hashing split over the peer mesh, on 2
and 4 GPUs: every rank's proof equals the one-GPU proof byte for byte, and the oracle's chain verifier accepts
it, for transformer blocks whose weight MLEs are large enough to split (skipped with fewer GPUs)."""
import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]
SHAPES = [(4, 64, 64, 128), (2, 256, 256, 512)]


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _case(i):
    sys.path[:0] = [str(ROOT / "tests"), str(ROOT / "stwo-ml_b200")]
    from helpers import int_matrix_m31
    from zkml_b200.circuits import hf_transformer_layers
    m, d, q, f = SHAPES[i]
    x = int_matrix_m31(m, d, 900 + i, bound=32767)
    layers = hf_transformer_layers(d, q, f, 1, lambda j, r, c: int_matrix_m31(r, c, 9000 + 10 * i + j), "silu")
    return x, layers


def _worker(rank, world, port, out_dir):
    sys.path[:0] = [str(ROOT), str(ROOT / "tests"), str(ROOT / "stwo-ml_b200")]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist
    import zkml_b200 as Z
    from zkml_b200.distributed import PeerMesh
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    mesh = PeerMesh(ctx=Z.context(rank))
    try:
        for i in range(len(SHAPES)):
            x, layers = _case(i)
            proof = Z.prove_gkr_chain(x, layers, n_queries=6, mesh=mesh, activation_logup=False)
            np.save(os.path.join(out_dir, f"r{rank}_c{i}.npy"), proof.raw)
        torch.cuda.synchronize()
        dist.barrier()
    finally:
        mesh.close()
        dist.destroy_process_group()


@pytest.mark.gpu
@pytest.mark.parametrize("world", [2, 4])
def test_mesh_chain_equals_one_gpu(world, tmp_path):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    mp.start_processes(_worker, args=(world, _port(), str(tmp_path)), nprocs=world, join=True, start_method="spawn")
    sys.path[:0] = [str(ROOT / "stwo-ml_b200"), str(ROOT / "tests")]
    import oracle_lib as O
    import zkml_b200 as Z
    for i in range(len(SHAPES)):
        x, layers = _case(i)
        ref = Z.prove_gkr_chain(x, layers, n_queries=6, activation_logup=False).raw
        assert O.verify_gkr_chain(x, layers, ref, n_queries=6, activation_logup=False)[0]
        for r in range(world):
            got = np.load(tmp_path / f"r{r}_c{i}.npy")
            assert got.size == ref.size and (got == ref).all(), (i, r)
