"""The library's shared-memory exchange (zkml_shm_exchange_*): host-only, CPU ranks."""
import os
import sys
import uuid
from pathlib import Path

import numpy as np
import pytest
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]


def _worker(rank, world, name, out_dir, nonce=None, delay_rank0=0.0):
    sys.path[:0] = [str(ROOT / "stwo-ml_b200")]
    import time
    from zkml_b200.distributed import ShmExchange
    if rank == 0 and delay_rank0:
        time.sleep(delay_rank0)
    ex = ShmExchange(name, world, rank, max_gather_bytes=1 << 16, nonce=nonce if nonce is not None else
                     int(name[-12:], 16))
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


def test_shm_stale_segment_of_an_earlier_job_is_not_joined(tmp_path):
    """A crashed job leaves a ready segment under the same name; the new job's rank 1
    opens the name before rank 0 has replaced it and must wait for its own nonce."""
    sys.path[:0] = [str(ROOT / "stwo-ml_b200")]
    from zkml_b200.distributed import ShmExchange
    name = "zkml_stale_" + uuid.uuid4().hex[:12]
    stale = ShmExchange(name, 2, 0, max_gather_bytes=1 << 16, nonce=1)
    try:
        stale.struct.allreduce_u64  # the stale job is left mapped and never closed
        mp.start_processes(_worker, args=(2, name, str(tmp_path), 2, 1.0), nprocs=2, join=True,
                           start_method="spawn")
        for rank in range(2):
            got = np.load(tmp_path / f"r{rank}.npz")
            for r in range(20):
                np.testing.assert_array_equal(got["sums"][r], np.arange(12, dtype=np.uint64) * 3 + 2 * r)
    finally:
        stale.close()
