"""One product sumcheck split across GPUs (one process per GPU).

The degree-2 product sumcheck that ``ZkmlOps::reduce_matmul_layer`` runs
(engine/src/backend.rs:141-178, round loop of components/matmul.rs
``prove_matmul_sumcheck_onchain``) is sharded by the low index bits: rank g of
G holds the elements whose global index i satisfies i = g (mod G), in order,
so local element j is global element j*G + g.  A fold pairs global i with
i + N/2; both are on the same rank at local j and j + N_loc/2, and the folded
value keeps global index i, so the layout survives every fold.  Each round's
(s0, s1, s2) is therefore the sum over ranks of the local sums: the only
exchange per round is 12 u32 words (an all-reduce mod p).  Every rank runs the
same host Poseidon channel on the same sums and draws the same challenge, so
no challenge broadcast is needed.  Once the local length falls to the gather
threshold, each rank exports its folded vectors, they are all-gathered and
interleaved back to global order, and every rank finishes the (now small)
sumcheck on its own GPU.  The proof is bit-identical to the single-GPU one.

The collective is ``torch.distributed`` (NCCL between GPUs; gloo for the CPU
tests of this orchestration).
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass
from typing import List, Optional

import numpy as np

from . import (M31_P as P, PoseidonChannel, RoundPoly, Context, GKRClaim, M31Matrix, MatMulReduction, _Buf, _check,
               _log2, _next_pow2, _qm31_ptr, as_qm31_array, context, lib)

ALLREDUCE_FN = C.CFUNCTYPE(C.c_int, C.c_void_p, C.POINTER(C.c_uint64), C.c_int)
ALLGATHER_FN = C.CFUNCTYPE(C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t)


class ExchangeStruct(C.Structure):
    """`zkml_exchange` of the C ABI."""
    _fields_ = [("user", C.c_void_p), ("allreduce_u64", ALLREDUCE_FN), ("allgather", ALLGATHER_FN),
                ("world", C.c_int), ("rank", C.c_int)]


def job_nonce(group=None) -> int:
    """A 64-bit value that is the same on every rank of the process group and new for each
    call: rank 0 draws it and broadcasts it (a single process draws its own)."""
    import secrets
    import torch
    import torch.distributed as dist
    v = secrets.randbits(63)
    if dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1:
        dev = "cuda" if dist.get_backend(group) == "nccl" else "cpu"
        t = torch.tensor([v], dtype=torch.int64, device=dev)
        dist.broadcast(t, src=dist.get_global_rank(group, 0) if group is not None else 0, group=group)
        v = int(t.item())
    return v


class ShmExchange:
    """The library's shared-memory exchange between the ranks (processes) of one node.

    `nonce` must be equal on all ranks and new per job (see `job_nonce`); it keeps a rank
    from joining a segment that an earlier job left under the same name."""

    def __init__(self, name: str, world: int, rank: int, max_gather_bytes: int = 64 << 20, *, nonce: int):
        self.struct = ExchangeStruct()
        _check(lib().zkml_shm_exchange_open(name.encode(), world, rank, max_gather_bytes, nonce & (2**64 - 1),
                                            C.byref(self.struct)))
        self.world, self.rank = world, rank

    def allreduce(self, words) -> np.ndarray:
        buf = np.ascontiguousarray(words, np.uint64).copy()
        _check(self.struct.allreduce_u64(self.struct.user, buf.ctypes.data_as(C.POINTER(C.c_uint64)), len(buf)))
        return buf

    def allgather(self, local: np.ndarray) -> np.ndarray:
        local = np.ascontiguousarray(local)
        out = np.empty((self.world,) + local.shape, local.dtype)
        _check(self.struct.allgather(self.struct.user, local.ctypes.data_as(C.c_void_p),
                                     out.ctypes.data_as(C.c_void_p), local.nbytes))
        return out

    def close(self) -> None:
        if self.struct.user:
            lib().zkml_shm_exchange_close(C.byref(self.struct))

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class TorchExchange:
    """A zkml_exchange whose two collectives are torch.distributed calls (NCCL or gloo)."""

    def __init__(self, group=None):
        import torch
        import torch.distributed as dist
        self.torch, self.dist, self.group = torch, dist, group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.device = (torch.device("cuda", torch.cuda.current_device()) if dist.get_backend(group) == "nccl"
                       else torch.device("cpu"))

        def allreduce(_user, words, n):
            try:
                arr = np.ctypeslib.as_array(words, shape=(n,))
                t = torch.from_numpy(arr.astype(np.int64)).to(self.device)
                dist.all_reduce(t, group=self.group)
                arr[:] = t.cpu().numpy().astype(np.uint64)
                return 0
            except Exception:
                return 4

        def allgather(_user, local, out, nbytes):
            try:
                src = np.ctypeslib.as_array(C.cast(local, C.POINTER(C.c_uint8)), shape=(nbytes,))
                t = torch.from_numpy(src.copy()).to(self.device)
                parts = [torch.empty_like(t) for _ in range(self.world)]
                dist.all_gather(parts, t, group=self.group)
                dst = np.ctypeslib.as_array(C.cast(out, C.POINTER(C.c_uint8)), shape=(nbytes * self.world,))
                for r, part in enumerate(parts):
                    dst[r * nbytes:(r + 1) * nbytes] = part.cpu().numpy()
                return 0
            except Exception:
                return 4

        self._fns = (ALLREDUCE_FN(allreduce), ALLGATHER_FN(allgather))  # keep alive
        self.struct = ExchangeStruct(None, self._fns[0], self._fns[1], self.world, self.rank)

    def close(self) -> None:
        pass


def prove_product_sharded_native(a_local, b_local, n: int, channel: PoseidonChannel, exchange,
                                 gather_local: Optional[int] = None, ctx: Optional[Context] = None
                                 ) -> "ShardedSumcheckProof":
    """The same proof as prove_product_sharded, with the round loop inside the library
    (zkml_prove_product_sharded); `exchange` is a ShmExchange or a TorchExchange.  By default
    the vectors are gathered when the global length reaches 2^17 (each rank then finishes
    on 2^17 elements, ~0.45 ms)."""
    ctx = ctx or context()
    if gather_local is None:
        gather_local = max(2, (1 << 17) // exchange.world)
    ab, bb = _Buf(a_local), _Buf(b_local)
    log_n = n.bit_length() - 1
    rp = np.zeros((max(log_n, 1), 12), np.uint32)
    ch = np.zeros((max(log_n, 1), 4), np.uint32)
    fa = np.zeros(4, np.uint32)
    fb = np.zeros(4, np.uint32)
    gathered = C.c_size_t(0)
    _check(lib().zkml_prove_product_sharded(ctx.handle, ab.ptr, bb.ptr, n, gather_local, C.byref(exchange.struct),
                                            C.byref(channel.state), rp.reshape(-1), ch.reshape(-1), fa, fb,
                                            C.byref(gathered)))
    polys = [RoundPoly(rp[r, 0:4].copy(), rp[r, 4:8].copy(), rp[r, 8:12].copy()) for r in range(log_n)]
    return ShardedSumcheckProof(polys, ch[:log_n].copy(), fa, fb, int(gathered.value))

class PeerMesh:
    """The library's peer-memory mesh (zkml_mesh_*): this rank's inbox in HBM, mapped by every
    rank of `group` through CUDA IPC handles exchanged over the process group.  The round words
    and the gather of the sharded product sumcheck then travel as peer stores over NVLink
    inside the library's kernels.  The ranks must be on distinct GPUs of one node.
    max_gather_bytes bounds one rank's share of a gather (32 x gather_local bytes)."""

    def __init__(self, group=None, ctx: Optional[Context] = None, max_gather_bytes: int = 32 << 17):
        import torch
        import torch.distributed as dist
        self.ctx = ctx or context(torch.cuda.current_device())
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        h = (C.c_uint8 * 64)()
        _check(lib().zkml_mesh_create(self.ctx.handle, self.world, self.rank, max_gather_bytes, h))
        hs, devs = [bytes(h)], [str(torch.cuda.get_device_properties(self.ctx.device).uuid)]
        if self.world > 1:
            devs = [None] * self.world
            dist.all_gather_object(devs, str(torch.cuda.get_device_properties(self.ctx.device).uuid), group=group)
            if len(set(devs)) != self.world:
                lib().zkml_mesh_close(self.ctx.handle)
                raise ValueError("PeerMesh ranks must be on distinct GPUs")
            hs = [None] * self.world
            dist.all_gather_object(hs, bytes(h), group=group)
        allh = (C.c_uint8 * (64 * self.world)).from_buffer_copy(b"".join(hs))
        _check(lib().zkml_mesh_open(self.ctx.handle, allh, self.world))
        if self.world > 1:
            dist.barrier(group=group)
        self.closed = False

    def close(self) -> None:
        if not self.closed:
            lib().zkml_mesh_close(self.ctx.handle)
            self.closed = True


def prove_product_sharded_mesh(a_local, b_local, n: int, channel: PoseidonChannel, mesh: PeerMesh,
                               gather_local: Optional[int] = None) -> "ShardedSumcheckProof":
    """prove_product_sharded_native with the exchange over the peer mesh
    (zkml_prove_product_sharded_mesh): each split round's words are added across the ranks
    inside the round kernel and the folded vectors are gathered by peer stores."""
    if gather_local is None:
        gather_local = max(2, (1 << 17) // mesh.world)
    ab, bb = _Buf(a_local), _Buf(b_local)
    log_n = n.bit_length() - 1
    rp = np.zeros((max(log_n, 1), 12), np.uint32)
    ch = np.zeros((max(log_n, 1), 4), np.uint32)
    fa = np.zeros(4, np.uint32)
    fb = np.zeros(4, np.uint32)
    gathered = C.c_size_t(0)
    _check(lib().zkml_prove_product_sharded_mesh(mesh.ctx.handle, ab.ptr, bb.ptr, n, gather_local,
                                                 C.byref(channel.state), rp.ctypes.data, ch.ctypes.data,
                                                 fa.ctypes.data, fb.ctypes.data, C.byref(gathered)))
    polys = [RoundPoly(rp[r, 0:4].copy(), rp[r, 4:8].copy(), rp[r, 8:12].copy()) for r in range(log_n)]
    return ShardedSumcheckProof(polys, ch[:log_n].copy(), fa, fb, int(gathered.value))


INV2 = (P + 1) // 2


def shard_of(x: np.ndarray, rank: int, world: int) -> np.ndarray:
    """Rank `rank`'s share of a length-N vector: elements rank, rank+G, rank+2G, ..."""
    return np.ascontiguousarray(x[rank::world])


def interpolate(words: np.ndarray):
    """(s0, s1, s2) -> coefficients (c0, c1, c2) of s(X) = c0 + c1 X + c2 X^2.

    s2 is the sum at X = 2: c2 = (s2 - 2 s1 + s0) / 2, c1 = s1 - s0 - c2
    (components/matmul.rs, degree-2 round polynomial from three evaluations).
    The map is linear with base-field coefficients, so it acts coordinate-wise.
    """
    w = np.asarray(words, np.int64).reshape(3, 4)
    s0, s1, s2 = w[0], w[1], w[2]
    c0 = s0 % P
    c2 = ((s2 - 2 * s1 + s0) % P) * INV2 % P
    c1 = (s1 - s0 - c2) % P
    return c0.astype(np.uint32), c1.astype(np.uint32), c2.astype(np.uint32)


class GpuSumcheckSession:
    """The stepwise product sumcheck of one context (zkml_sumcheck_* in the C ABI)."""

    def __init__(self, ctx: Optional[Context] = None, device: int = 0):
        self.ctx = ctx or context(device)

    def load_m31(self, a, b) -> None:
        ab, bb = _Buf(a), _Buf(b)
        n = ab.nbytes // 4
        if bb.nbytes != ab.nbytes:
            raise ValueError("vectors differ in length")
        self._keep = (ab, bb)
        _check(lib().zkml_sumcheck_load_m31(self.ctx.handle, ab.ptr, bb.ptr, n))

    def load_qm31(self, a, b) -> None:
        ab, bb = _Buf(a), _Buf(b)
        n = ab.nbytes // 16
        if bb.nbytes != ab.nbytes:
            raise ValueError("vectors differ in length")
        self._keep = (ab, bb)
        _check(lib().zkml_sumcheck_load_qm31(self.ctx.handle, ab.ptr, bb.ptr, n))

    def length(self) -> int:
        return int(lib().zkml_sumcheck_length(self.ctx.handle))

    def round(self, alpha=None) -> np.ndarray:
        out = np.zeros(12, np.uint32)
        if alpha is None:
            _check(lib().zkml_sumcheck_round(self.ctx.handle, None, out))
        else:
            al = np.ascontiguousarray(alpha, np.uint32).reshape(4)
            _check(lib().zkml_sumcheck_round(self.ctx.handle, al.ctypes.data_as(C.c_void_p), out))
        return out

    def export(self):
        n = self.length()
        a = np.zeros((n, 4), np.uint32)
        b = np.zeros((n, 4), np.uint32)
        _check(lib().zkml_sumcheck_export(self.ctx.handle, a.ctypes.data_as(C.c_void_p),
                                          b.ctypes.data_as(C.c_void_p)))
        return a, b

    def finalize(self, alpha):
        fa = np.zeros(4, np.uint32)
        fb = np.zeros(4, np.uint32)
        _check(lib().zkml_sumcheck_finalize(self.ctx.handle, np.ascontiguousarray(alpha, np.uint32).reshape(4),
                                            fa, fb))
        return fa, fb


class LocalCollective:
    """World size 1: the whole product on this process's GPU."""

    world, rank = 1, 0

    def sum_words(self, words):
        return words

    def gather_interleaved(self, local):
        return local

    def gather_interleaved_m31(self, local):
        return local


class TorchCollective:
    """The two exchanges of the sharded sumcheck over a torch.distributed group."""

    def __init__(self, group=None):
        import torch
        import torch.distributed as dist
        self.torch, self.dist, self.group = torch, dist, group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if dist.get_backend(group) == "nccl":
            self.device = torch.device("cuda", torch.cuda.current_device())
        else:
            self.device = torch.device("cpu")

    def sum_words(self, words: np.ndarray) -> np.ndarray:
        t = self.torch.from_numpy(np.asarray(words, np.int64).copy()).to(self.device)
        self.dist.all_reduce(t, group=self.group)
        return (t.cpu().numpy() % P).astype(np.uint32)

    def gather_interleaved(self, local: np.ndarray) -> np.ndarray:
        """All-gather the (L, 4) local vectors and return the (L*G, 4) global one."""
        t = self.torch.from_numpy(local.view(np.int32).copy()).to(self.device)
        parts = [self.torch.empty_like(t) for _ in range(self.world)]
        self.dist.all_gather(parts, t, group=self.group)
        stacked = np.stack([p.cpu().numpy().view(np.uint32) for p in parts])  # (G, L, 4)
        return np.ascontiguousarray(stacked.transpose(1, 0, 2).reshape(-1, 4))

    def gather_interleaved_m31(self, local: np.ndarray) -> np.ndarray:
        t = self.torch.from_numpy(np.asarray(local, np.uint32).view(np.int32).copy()).to(self.device)
        parts = [self.torch.empty_like(t) for _ in range(self.world)]
        self.dist.all_gather(parts, t, group=self.group)
        stacked = np.stack([p.cpu().numpy().view(np.uint32) for p in parts])  # (G, L)
        return np.ascontiguousarray(stacked.T.reshape(-1))


@dataclass
class ShardedSumcheckProof:
    round_polys: List[RoundPoly]
    challenges: np.ndarray   # (log N, 4)
    final_a: np.ndarray
    final_b: np.ndarray
    gathered_at: int         # global length at which the vectors were gathered (N if never sharded)


DEFAULT_GATHER_LOCAL = 1 << 16


def prove_product_sharded(a_local, b_local, n: int, channel: PoseidonChannel, session=None, collective=None,
                          gather_local: int = DEFAULT_GATHER_LOCAL) -> ShardedSumcheckProof:
    """Prove sum_i a_i b_i over a length-n M31 product split across the group.

    a_local, b_local: this rank's shares (``shard_of``) of the two M31 vectors,
    each of length n / G (host arrays or device tensors).  Every rank returns
    the same proof, equal to the single-GPU ``reduce_matmul_layer`` on the 1 x n
    and n x 1 matrices (no restriction point).  `gather_local` is the local
    length at or below which the vectors are gathered onto every GPU.
    """
    session = session or GpuSumcheckSession()
    col = collective or TorchCollective()
    G = col.world
    if n < 2 or n & (n - 1):
        raise ValueError("n must be a power of two >= 2")
    if G & (G - 1) or n % G:
        raise ValueError("world size must be a power of two dividing n")
    n_loc = n // G
    log_n = n.bit_length() - 1
    sharded = G > 1 and n_loc >= 4 and n_loc > gather_local
    gathered_at = n
    if sharded:
        session.load_m31(a_local, b_local)
    elif G > 1:
        # too small to split: every rank proves the whole vector
        a_host = np.asarray(a_local.cpu() if hasattr(a_local, "cpu") else a_local, np.uint32)
        b_host = np.asarray(b_local.cpu() if hasattr(b_local, "cpu") else b_local, np.uint32)
        session.load_m31(col.gather_interleaved_m31(a_host), col.gather_interleaved_m31(b_host))
    else:
        session.load_m31(a_local, b_local)
    sums = session.round(None)
    glen = n
    polys: List[RoundPoly] = []
    chals = np.zeros((log_n, 4), np.uint32)
    final_a = final_b = None
    for r in range(log_n):
        if sharded:
            sums = col.sum_words(sums)
        c0, c1, c2 = interpolate(sums)
        channel.mix_poly_coeffs(c0, c1, c2)
        alpha = channel.draw_qm31()
        polys.append(RoundPoly(c0, c1, c2))
        chals[r] = alpha
        if glen == 2:
            final_a, final_b = session.finalize(alpha)
            break
        sums = session.round(alpha)
        glen //= 2
        if sharded and glen // G <= max(gather_local, 2):
            la, lb = session.export()
            session.load_qm31(col.gather_interleaved(la), col.gather_interleaved(lb))
            sharded = False
            gathered_at = glen
            sums = session.round(None)
    return ShardedSumcheckProof(polys, chals, final_a, final_b, gathered_at)


# ---------------------------------------------------------------------------
# One matmul layer split by column blocks of the weight
# ---------------------------------------------------------------------------

def column_block(n: int, rank: int, world: int):
    """Columns [lo, hi) of B that `rank` holds: the padded column space next_pow2(n) cut into
    `world` equal blocks (each a multiple of 64 columns), clipped to the n real columns
    (a rank whose block is all padding holds none: lo == hi)."""
    pn = _next_pow2(n)
    block = pn // world
    if block * world != pn or block % 64:
        raise ValueError(f"next_pow2(n) = {pn} does not split into {world} blocks of a multiple of 64 columns")
    lo = min(rank * block, n)
    return lo, min(lo + block, n) if lo < n else lo


def restrict_cols_block_words(b_block, k: int, col_offset: int, r_j, ctx: Optional[Context] = None):
    """This rank's 4k partial words of f_b (a CUDA int64 tensor): its column block restricted
    with the weights of the full padded column space (zkml_restrict_cols_block)."""
    import torch
    ctx = ctx or context(torch.cuda.current_device())
    words = torch.zeros(4 * k, dtype=torch.int64, device=torch.device("cuda", ctx.device))
    bm = b_block if isinstance(b_block, M31Matrix) else None
    n_block = bm.cols if bm is not None else (int(b_block.shape[1]) if b_block is not None else 0)
    if n_block:
        bb = _Buf(bm.data if bm is not None else b_block)
        rj = np.ascontiguousarray(as_qm31_array(r_j), np.uint32)
        _check(lib().zkml_restrict_cols_block(ctx.handle, bb.ptr, k, n_block, col_offset,
                                              rj.ctypes.data_as(C.c_void_p) if rj.size else None, len(rj),
                                              C.c_void_p(words.data_ptr())))
    return words


def reduce_matmul_layer_from_words(output_claim: GKRClaim, a: M31Matrix, words, m: int, k: int, n: int,
                                   channel: PoseidonChannel, ctx: Optional[Context] = None):
    """The layer from the all-reduced partial words (zkml_reduce_matmul_layer_gkr_fb)."""
    import torch
    ctx = ctx or context(torch.cuda.current_device())
    pm, pk, pn = _next_pow2(m), _next_pow2(k), _next_pow2(n)
    log_m, log_k = _log2(pm), _log2(pk)
    point = as_qm31_array(output_claim.point)
    ab = _Buf(a.data)
    pt_ptr, pt_keep = _qm31_ptr(point)
    rp = np.zeros((max(log_k, 1), 12), np.uint32)
    fa = np.zeros(4, np.uint32)
    fb = np.zeros(4, np.uint32)
    nxt = np.zeros((max(log_m + log_k, 1), 4), np.uint32)
    _check(lib().zkml_reduce_matmul_layer_gkr_fb(ctx.handle, pt_ptr, len(point),
                                                 np.ascontiguousarray(output_claim.value, np.uint32).reshape(4),
                                                 ab.ptr, m, k, C.c_void_p(words.data_ptr()), n,
                                                 C.byref(channel.state), rp.reshape(-1), fa, fb, nxt.reshape(-1)))
    polys = [RoundPoly(rp[r, 0:4].copy(), rp[r, 4:8].copy(), rp[r, 8:12].copy()) for r in range(log_k)]
    red = MatMulReduction(polys, nxt[log_m:log_m + log_k].copy(), fa, fb)
    return red, GKRClaim(nxt[:log_m + log_k].copy(), fa.copy())


def reduce_matmul_layer_colsharded(output_claim: GKRClaim, a: M31Matrix, b_block, col_offset: int, m: int, k: int,
                                   n: int, channel: PoseidonChannel, group=None, ctx: Optional[Context] = None):
    """reduce_matmul_layer_with_backend (gkr/prover.rs:5959-6073) for a layer whose weight is
    split by column blocks over the ranks of `group` (one GPU each; rank g holds
    B[:, column_block(n, g, world)] as `b_block`, k x (hi - lo), device or host memory).
    Each rank restricts its block; one NCCL all-reduce adds the 4k partial words; every rank
    then runs the (small) sumcheck from the sum and returns the same reduction and next
    claim as the unsplit layer."""
    import torch.distributed as dist
    pm, pn = _next_pow2(m), _next_pow2(n)
    point = as_qm31_array(output_claim.point)
    if len(point) != _log2(pm) + _log2(pn):
        raise ValueError("output claim must have log2(pm) + log2(pn) variables")
    words = restrict_cols_block_words(b_block, k, col_offset, point[_log2(pm):], ctx)
    if dist.is_initialized() and dist.get_world_size(group) > 1:
        dist.all_reduce(words, group=group)
    return reduce_matmul_layer_from_words(output_claim, a, words, m, k, n, channel, ctx)


class P2PInbox:
    """The peer-memory exchange of the split layer (zkml_p2p_*): this rank's inbox for the
    layer's k, mapped by every rank of `group` (CUDA IPC handles exchanged through the
    process group).  The ranks must be on distinct GPUs of one node."""

    def __init__(self, k: int, group=None, ctx: Optional[Context] = None):
        import torch
        import torch.distributed as dist
        self.ctx = ctx or context(torch.cuda.current_device())
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.k = k
        self.epoch = 0
        h = (C.c_uint8 * 64)()
        _check(lib().zkml_p2p_inbox_create(self.ctx.handle, k, self.world, self.rank, h))
        devs = [None] * self.world
        dist.all_gather_object(devs, str(torch.cuda.get_device_properties(self.ctx.device).uuid), group=group)
        if len(set(str(d) for d in devs)) != self.world:
            lib().zkml_p2p_close(self.ctx.handle)
            raise ValueError("P2PInbox ranks must be on distinct GPUs")
        hs = [None] * self.world
        dist.all_gather_object(hs, bytes(h), group=group)
        allh = (C.c_uint8 * (64 * self.world)).from_buffer_copy(b"".join(hs))
        _check(lib().zkml_p2p_open(self.ctx.handle, allh, self.world))
        dist.barrier(group=group)

    def close(self) -> None:
        lib().zkml_p2p_close(self.ctx.handle)


def reduce_matmul_layer_colsharded_p2p(output_claim: GKRClaim, a: M31Matrix, b_block, col_offset: int, m: int, k: int,
                                       n: int, channel: PoseidonChannel, inbox: P2PInbox):
    """reduce_matmul_layer_colsharded with the exchange over peer memory: the block
    restriction's partial words go straight into every rank's inbox (no collective library,
    no host step between the two kernels)."""
    pm, pn = _next_pow2(m), _next_pow2(n)
    log_m, log_k = _log2(pm), _log2(_next_pow2(k))
    point = as_qm31_array(output_claim.point)
    if len(point) != log_m + _log2(pn):
        raise ValueError("output claim must have log2(pm) + log2(pn) variables")
    ctx = inbox.ctx
    inbox.epoch += 1
    bm = b_block if isinstance(b_block, M31Matrix) else None
    n_block = bm.cols if bm is not None else (int(b_block.shape[1]) if b_block is not None else 0)
    bb = _Buf(bm.data if bm is not None else b_block) if n_block else None
    rj = np.ascontiguousarray(point[log_m:], np.uint32)
    _check(lib().zkml_restrict_cols_block_p2p(ctx.handle, bb.ptr if bb else None, k, n_block, col_offset,
                                              rj.ctypes.data_as(C.c_void_p) if rj.size else None, len(rj),
                                              inbox.epoch))
    ab = _Buf(a.data)
    pt_ptr, pt_keep = _qm31_ptr(point)
    rp = np.zeros((max(log_k, 1), 12), np.uint32)
    fa = np.zeros(4, np.uint32)
    fb = np.zeros(4, np.uint32)
    nxt = np.zeros((max(log_m + log_k, 1), 4), np.uint32)
    _check(lib().zkml_reduce_matmul_layer_gkr_p2p(ctx.handle, pt_ptr, len(point),
                                                  np.ascontiguousarray(output_claim.value, np.uint32).reshape(4),
                                                  ab.ptr, m, k, n, inbox.epoch, C.byref(channel.state),
                                                  rp.reshape(-1), fa, fb, nxt.reshape(-1)))
    polys = [RoundPoly(rp[r, 0:4].copy(), rp[r, 4:8].copy(), rp[r, 8:12].copy()) for r in range(log_k)]
    red = MatMulReduction(polys, nxt[log_m:log_m + log_k].copy(), fa, fb)
    return red, GKRClaim(nxt[:log_m + log_k].copy(), fa.copy())
