"""The product sumcheck split across ranks equals the single-device proof.

CPU: world-size 2 and 4 gloo ranks drive a numpy double of the GPU session;
GPU: two gloo ranks share cuda:0, each driving its own context through the
C ABI (the exchange is host-side, so the ranks never wait on one another
inside a kernel).  Both are checked against the oracle's reduce_matmul_layer
on the 1 x N and N x 1 matrices.
"""
import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest
import torch.multiprocessing as mp

import oracle_lib
from helpers import uniform_m31

ROOT = Path(__file__).resolve().parents[1]


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, n, gather_local, use_gpu, out_dir):
    sys.path[:0] = [str(ROOT), str(ROOT / "tests"), str(ROOT / "stwo-ml_b200")]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch.distributed as dist
    from zkml_b200 import PoseidonChannel
    from zkml_b200.distributed import GpuSumcheckSession, prove_product_sharded, shard_of
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        a = uniform_m31(n, 11)
        b = uniform_m31(n, 12)
        if use_gpu:
            session = GpuSumcheckSession(device=0)
        else:
            from sumcheck_double import NumpySumcheckSession
            session = NumpySumcheckSession()
        proof = prove_product_sharded(shard_of(a, rank, world), shard_of(b, rank, world), n, PoseidonChannel(),
                                      session=session, gather_local=gather_local)
        rp = np.stack([np.concatenate([p.c0, p.c1, p.c2]) for p in proof.round_polys])
        np.savez(os.path.join(out_dir, f"r{rank}.npz"), rp=rp, ch=proof.challenges, fa=proof.final_a,
                 fb=proof.final_b, gathered=proof.gathered_at)
    finally:
        dist.destroy_process_group()


def _native_worker(rank, world, name, n, gather_local, out_dir):
    sys.path[:0] = [str(ROOT), str(ROOT / "tests"), str(ROOT / "stwo-ml_b200")]
    from zkml_b200 import PoseidonChannel
    from zkml_b200.distributed import ShmExchange, prove_product_sharded_native, shard_of
    ex = ShmExchange(name, world, rank, max_gather_bytes=max(1 << 16, 32 * (n // world)), nonce=int(name[-12:], 16))
    try:
        a = uniform_m31(n, 11)
        b = uniform_m31(n, 12)
        proof = prove_product_sharded_native(shard_of(a, rank, world), shard_of(b, rank, world), n, PoseidonChannel(),
                                             ex, gather_local=gather_local)
        rp = np.stack([np.concatenate([p.c0, p.c1, p.c2]) for p in proof.round_polys])
        np.savez(os.path.join(out_dir, f"r{rank}.npz"), rp=rp, ch=proof.challenges, fa=proof.final_a,
                 fb=proof.final_b, gathered=proof.gathered_at)
    finally:
        ex.close()


def _check_against_oracle(world, n, tmp_path):
    a = uniform_m31(n, 11)
    b = uniform_m31(n, 12)
    ref = oracle_lib.reduce_matmul_layer(a.reshape(1, n), b.reshape(n, 1), np.zeros((0, 4), np.uint32),
                                         np.zeros((0, 4), np.uint32), oracle_lib.new_channel(), mode=0, nthreads=4)
    gathered = []
    for r in range(world):
        got = np.load(tmp_path / f"r{r}.npz")
        np.testing.assert_array_equal(got["rp"], ref["round_polys"])
        np.testing.assert_array_equal(got["ch"], ref["challenges"])
        np.testing.assert_array_equal(got["fa"], ref["final_a"])
        np.testing.assert_array_equal(got["fb"], ref["final_b"])
        gathered.append(int(got["gathered"]))
    return gathered


@pytest.mark.gpu
@pytest.mark.parametrize("world,n,gather_local", [(2, 1 << 16, 1 << 8), (2, 1 << 12, 2), (4, 1 << 14, 1 << 6),
                                                  (2, 1 << 6, 1 << 16)])
def test_native_sharded_matches_oracle_gpu(world, n, gather_local, tmp_path):
    """The library's round loop (zkml_prove_product_sharded) with the shared-memory exchange, ranks on one GPU."""
    import uuid
    name = "zkml_t_" + uuid.uuid4().hex[:12]
    mp.start_processes(_native_worker, args=(world, name, n, gather_local, str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    gathered = _check_against_oracle(world, n, tmp_path)
    if n // world > max(gather_local, 2):
        assert gathered[0] < n


def _run(world, n, gather_local, use_gpu, tmp_path):
    mp.start_processes(_worker, args=(world, _free_port(), n, gather_local, use_gpu, str(tmp_path)), nprocs=world,
                       join=True, start_method="spawn")
    a = uniform_m31(n, 11)
    b = uniform_m31(n, 12)
    ref = oracle_lib.reduce_matmul_layer(a.reshape(1, n), b.reshape(n, 1), np.zeros((0, 4), np.uint32),
                                         np.zeros((0, 4), np.uint32), oracle_lib.new_channel(), mode=0, nthreads=1)
    gathered = []
    for r in range(world):
        got = np.load(tmp_path / f"r{r}.npz")
        np.testing.assert_array_equal(got["rp"], ref["round_polys"])
        np.testing.assert_array_equal(got["ch"], ref["challenges"])
        np.testing.assert_array_equal(got["fa"], ref["final_a"])
        np.testing.assert_array_equal(got["fb"], ref["final_b"])
        gathered.append(int(got["gathered"]))
    return gathered


@pytest.mark.parametrize("world,n,gather_local", [(2, 1 << 10, 16), (4, 1 << 9, 1), (2, 8, 1), (4, 16, 64)])
def test_sharded_matches_oracle_cpu(world, n, gather_local, tmp_path):
    gathered = _run(world, n, gather_local, False, tmp_path)
    if n // world > gather_local and n // world >= 4:
        assert gathered[0] < n  # the split path was taken


def test_interpolate_matches_channel_coefficients():
    from zkml_b200.distributed import interpolate
    rng = np.random.default_rng(5)
    s = rng.integers(0, oracle_lib.P if hasattr(oracle_lib, "P") else (1 << 31) - 1, 12, dtype=np.int64)
    c0, c1, c2 = (x.astype(np.int64) for x in interpolate(s))
    p = (1 << 31) - 1
    s0, s1, s2 = s[:4], s[4:8], s[8:]
    np.testing.assert_array_equal(c0 % p, s0 % p)
    np.testing.assert_array_equal((c0 + c1 + c2) % p, s1 % p)
    np.testing.assert_array_equal((c0 + 2 * c1 + 4 * c2) % p, s2 % p)


@pytest.mark.gpu
@pytest.mark.parametrize("n,gather_local", [(1 << 16, 1 << 8), (1 << 12, 2)])
def test_sharded_matches_oracle_gpu(n, gather_local, tmp_path):
    gathered = _run(2, n, gather_local, True, tmp_path)
    assert gathered[0] < n


def _single_gpu_proof(a, b):
    from zkml_b200 import PoseidonChannel
    from zkml_b200.distributed import GpuSumcheckSession, LocalCollective, prove_product_sharded
    return prove_product_sharded(a, b, len(a), PoseidonChannel(), session=GpuSumcheckSession(),
                                 collective=LocalCollective())


def _oracle_proof(a, b):
    n = len(a)
    return oracle_lib.reduce_matmul_layer(np.asarray(a, np.uint32).reshape(1, n), np.asarray(b, np.uint32).reshape(n, 1),
                                          np.zeros((0, 4), np.uint32), np.zeros((0, 4), np.uint32),
                                          oracle_lib.new_channel(), mode=0, nthreads=1)


@pytest.mark.gpu
@pytest.mark.parametrize("kind", ["max", "zero", "p", "mixed", "uniform"])
def test_stepwise_edge_values_gpu(kind):
    """Field-edge inputs through the stepwise session (the lazy-reduction bounds)."""
    p = (1 << 31) - 1
    n = 1 << 14
    rng = np.random.default_rng(3)
    if kind == "max":
        a = np.full(n, p - 1, np.uint32); b = np.full(n, p - 1, np.uint32)
    elif kind == "zero":
        a = np.zeros(n, np.uint32); b = uniform_m31(n, 5)
    elif kind == "p":  # the non-canonical encoding of zero
        a = np.full(n, p, np.uint32); b = np.full(n, p - 1, np.uint32)
    elif kind == "mixed":
        a = rng.choice(np.array([0, 1, p - 1, p - 2, 1 << 30], np.uint32), n)
        b = rng.choice(np.array([0, 1, p - 1, p - 2, (1 << 30) + 1], np.uint32), n)
    else:
        a = uniform_m31(n, 7); b = uniform_m31(n, 8)
    got = _single_gpu_proof(a, b)
    ref = _oracle_proof(a, b)
    rp = np.stack([np.concatenate([q.c0, q.c1, q.c2]) for q in got.round_polys])
    np.testing.assert_array_equal(rp, ref["round_polys"])
    np.testing.assert_array_equal(got.challenges, ref["challenges"])
    np.testing.assert_array_equal(got.final_a, ref["final_a"])
    np.testing.assert_array_equal(got.final_b, ref["final_b"])


@pytest.mark.gpu
def test_stepwise_load_qm31_reduces_words_gpu():
    """load_qm31 accepts any u32 words and treats them mod p."""
    from zkml_b200.distributed import GpuSumcheckSession
    p = (1 << 31) - 1
    rng = np.random.default_rng(9)
    a = rng.integers(0, 1 << 32, (1 << 10, 4), dtype=np.uint64).astype(np.uint32)
    b = rng.integers(0, 1 << 32, (1 << 10, 4), dtype=np.uint64).astype(np.uint32)
    s1 = GpuSumcheckSession()
    s1.load_qm31(a, b)
    w1 = s1.round(None)
    s1.load_qm31((a.astype(np.uint64) % p).astype(np.uint32), (b.astype(np.uint64) % p).astype(np.uint32))
    w2 = s1.round(None)
    np.testing.assert_array_equal(w1, w2)
    ea, eb = s1.export()
    assert (ea < p).all() and (eb < p).all()
