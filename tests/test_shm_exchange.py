"""The library's shared-memory exchange (zkml_shm_exchange_*): host-only, CPU ranks."""
import os
import sys
import uuid
from pathlib import Path

import numpy as np
import pytest
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]


def _worker(rank, world, name, out_dir):
    sys.path[:0] = [str(ROOT / "stwo-ml_b200")]
    from zkml_b200.distributed import ShmExchange
    ex = ShmExchange(name, world, rank, max_gather_bytes=1 << 16)
    try:
        sums = [ex.allreduce(np.arange(12, dtype=np.uint64) * (rank + 1) + r) for r in range(20)]
        gathers = [ex.allgather(np.full(100 + r, rank * 1000 + r, np.uint32)) for r in range(3)]
        np.savez(os.path.join(out_dir, f"r{rank}.npz"), sums=np.stack(sums), g0=gathers[0], g1=gathers[1], g2=gathers[2])
    finally:
        ex.close()


@pytest.mark.parametrize("world", [1, 2, 4])
def test_shm_allreduce_allgather(world, tmp_path):
    name = "zkml_test_" + uuid.uuid4().hex[:12]
    mp.start_processes(_worker, args=(world, name, str(tmp_path)), nprocs=world, join=True, start_method="spawn")
    tri = world * (world + 1) // 2
    for rank in range(world):
        got = np.load(tmp_path / f"r{rank}.npz")
        for r in range(20):
            np.testing.assert_array_equal(got["sums"][r], np.arange(12, dtype=np.uint64) * tri + world * r)
        for r in range(3):
            g = got[f"g{r}"]
            assert g.shape == (world, 100 + r)
            for q in range(world):
                assert (g[q] == q * 1000 + r).all()
