"""Weight commitment cache, file-compatible with the engine's weight_cache.rs.

Weight matrices are fixed per model, so their Poseidon Merkle roots (and the restricted
weight MLEs of a given transcript) need computing once.  The cache maps
(node_id, m_padded, k_padded, n_padded) to a cached entry; full-weight MLE roots, used by
the aggregated weight binding, are stored under the sentinel m_padded = 0
(weight_cache.rs:283-328).

File format (weight_cache.rs:16-23, 337-526; version 4 written, 1-4 read), little endian:
    b"SWCF" | version u32 | model_id_len u32 | model_id (UTF-8) | fingerprint 32 B (v4)
    | entry_count u32 | entries
    entry: node_id u64 | m u64 | k u64 | n u64 | f_b (len u32, QM31 as 4 x u32 each)
           | b_commitment (32 B big endian) | r_j (len u32, QM31 ...)
           | [v2] root flag u8 (+ 32 B big-endian felt) | [v3] path flag u8 (+ len u32 + UTF-8)
The fingerprint (weight_cache.rs:646-683) is an FNV-1a style mix of each weight's node id,
shape and 8 evenly spaced samples into four 64-bit lanes.
"""
from __future__ import annotations

import os
import struct
from dataclasses import dataclass, field
from typing import Dict, Iterable, List, Optional, Tuple

import numpy as np

MAGIC = b"SWCF"
CACHE_VERSION = 4
MAX_MODEL_ID_LEN = 1024
MAX_ENTRIES = 100_000
MAX_SECUREFIELD_VEC_LEN = 1_000_000
MAX_PATH_LEN = 4096
FINGERPRINT_SAMPLES_PER_MATRIX = 8
_FNV_OFFSET = 0xCBF29CE484222325
_FNV_PRIME = 0x00000100000001B3
_M64 = (1 << 64) - 1


@dataclass
class CachedWeight:
    f_b: np.ndarray = field(default_factory=lambda: np.zeros((0, 4), np.uint32))  # restricted weight MLE
    b_commitment: int = 0
    r_j: np.ndarray = field(default_factory=lambda: np.zeros((0, 4), np.uint32))
    initial_mle_root: Optional[int] = None
    merkle_tree_cache_path: Optional[str] = None


def compute_weight_fingerprint(weights: Iterable[Tuple[int, np.ndarray]]) -> bytes:
    """compute_weight_fingerprint over (node_id, matrix) pairs in the model's order."""
    state = [_FNV_OFFSET] * 4
    for node_id, matrix in weights:
        m = np.asarray(matrix)
        data = m.reshape(-1)
        n = data.size
        if n == 0:
            continue
        rows, cols = (m.shape[0], m.shape[1]) if m.ndim == 2 else (1, n)
        state[0] = ((state[0] * _FNV_PRIME) & _M64) ^ node_id
        state[1] = ((state[1] * _FNV_PRIME) & _M64) ^ rows
        state[2] = ((state[2] * _FNV_PRIME) & _M64) ^ cols
        state[3] = ((state[3] * _FNV_PRIME) & _M64) ^ n
        step = max(1, n // FINGERPRINT_SAMPLES_PER_MATRIX)
        for i in range(min(FINGERPRINT_SAMPLES_PER_MATRIX, n)):
            val = int(data[min(i * step, n - 1)]) & 0xFFFFFFFF
            lane = i % 4
            state[lane] = ((state[lane] * _FNV_PRIME) & _M64) ^ val
    return b"".join(struct.pack("<Q", s) for s in state)


class WeightCommitmentCache:
    """In-memory cache of one model's weight commitments (weight_cache.rs:131-330)."""

    def __init__(self, model_id: str, fingerprint: bytes = bytes(32)):
        self.model_id = model_id
        self.fingerprint = fingerprint
        self.entries: Dict[Tuple[int, int, int, int], CachedWeight] = {}
        self.dirty = False
        self.auto_save_path: Optional[str] = None

    # -- entries -------------------------------------------------------------------
    def get(self, node_id: int, m_padded: int, k_padded: int, n_padded: int) -> Optional[CachedWeight]:
        return self.entries.get((node_id, m_padded, k_padded, n_padded))

    def insert(self, node_id: int, m_padded: int, k_padded: int, n_padded: int, entry: CachedWeight) -> None:
        self.entries[(node_id, m_padded, k_padded, n_padded)] = entry
        self.dirty = True

    def get_root(self, node_id: int, rows_padded: int, cols_padded: int) -> Optional[int]:
        e = self.entries.get((node_id, 0, rows_padded, cols_padded))
        return None if e is None else e.initial_mle_root

    def insert_root(self, node_id: int, rows_padded: int, cols_padded: int, root: int) -> None:
        self.entries[(node_id, 0, rows_padded, cols_padded)] = CachedWeight(initial_mle_root=root)
        self.dirty = True

    def __len__(self) -> int:
        return len(self.entries)

    def clear(self) -> None:
        self.entries.clear()
        self.dirty = True

    def set_fingerprint(self, fp: bytes) -> None:
        if fp != self.fingerprint:
            self.fingerprint = fp
            self.dirty = True

    def validate_fingerprint(self, weights: Iterable[Tuple[int, np.ndarray]]) -> bool:
        """A zero fingerprint (no validation) always matches (weight_cache.rs:266-281)."""
        if self.fingerprint == bytes(32):
            return True
        return self.fingerprint == compute_weight_fingerprint(weights)

    def root_for(self, node_id: int, weight, commit) -> int:
        """The weight's full-MLE root from the cache, or `commit(weight)` stored under it."""
        w = np.asarray(weight) if not hasattr(weight, "is_cuda") else weight
        rows, cols = int(w.shape[0]), int(w.shape[1])
        rp, cp = 1 << max(0, (rows - 1).bit_length()), 1 << max(0, (cols - 1).bit_length())
        root = self.get_root(node_id, rp, cp)
        if root is None:
            root = commit(weight)
            self.insert_root(node_id, rp, cp, root)
        return root

    # -- files ---------------------------------------------------------------------
    def save(self, path: str) -> None:
        if os.path.islink(path):
            raise PermissionError(f"Refusing to follow symlink: {path}")
        out = bytearray()
        out += MAGIC + struct.pack("<I", CACHE_VERSION)
        mid = self.model_id.encode()
        out += struct.pack("<I", len(mid)) + mid
        out += self.fingerprint
        out += struct.pack("<I", len(self.entries))
        for key in sorted(self.entries):
            e = self.entries[key]
            out += struct.pack("<4Q", *key)
            out += _sf_vec(e.f_b)
            out += e.b_commitment.to_bytes(32, "big")
            out += _sf_vec(e.r_j)
            if e.initial_mle_root is None:
                out += b"\x00"
            else:
                out += b"\x01" + e.initial_mle_root.to_bytes(32, "big")
            if e.merkle_tree_cache_path is None:
                out += b"\x00"
            else:
                pb = e.merkle_tree_cache_path.encode()
                out += b"\x01" + struct.pack("<I", len(pb)) + pb
        with open(path, "wb") as f:
            f.write(bytes(out))
        self.dirty = False

    @classmethod
    def load(cls, path: str) -> "WeightCommitmentCache":
        if os.path.islink(path):
            raise PermissionError(f"Refusing to follow symlink: {path}")
        with open(path, "rb") as f:
            r = _Reader(f.read())
        if r.take(4) != MAGIC:
            raise ValueError("not a weight cache file")
        version = r.u32()
        if not 1 <= version <= CACHE_VERSION:
            raise ValueError(f"unsupported cache version {version}, expected 1..={CACHE_VERSION}")
        id_len = r.u32()
        if id_len > MAX_MODEL_ID_LEN:
            raise ValueError(f"model_id length {id_len} exceeds maximum {MAX_MODEL_ID_LEN}")
        model_id = r.take(id_len).decode()
        fingerprint = r.take(32) if version >= 4 else bytes(32)
        n = r.u32()
        if n > MAX_ENTRIES:
            raise ValueError(f"entry count {n} exceeds maximum {MAX_ENTRIES}")
        cache = cls(model_id, fingerprint)
        for _ in range(n):
            key = tuple(r.u64() for _ in range(4))
            f_b = r.sf_vec()
            b_commitment = int.from_bytes(r.take(32), "big")
            r_j = r.sf_vec()
            root = None
            if version >= 2 and r.take(1) != b"\x00":
                root = int.from_bytes(r.take(32), "big")
            path_s = None
            if version >= 3 and r.take(1) != b"\x00":
                pl = r.u32()
                if pl > MAX_PATH_LEN:
                    raise ValueError(f"merkle_tree_cache_path length {pl} exceeds maximum {MAX_PATH_LEN}")
                path_s = r.take(pl).decode()
            cache.entries[key] = CachedWeight(f_b, b_commitment, r_j, root, path_s)
        cache.auto_save_path = path
        return cache

    @classmethod
    def load_or_new(cls, path: str, model_id: str) -> "WeightCommitmentCache":
        """The file's cache if it loads and belongs to model_id, else an empty one that saves there."""
        try:
            c = cls.load(path)
            if c.model_id == model_id:
                return c
        except (OSError, ValueError, struct.error):
            pass
        c = cls(model_id)
        c.auto_save_path = path
        return c

    def auto_save(self) -> None:
        if self.dirty and self.auto_save_path:
            self.save(self.auto_save_path)


def _sf_vec(v) -> bytes:
    a = np.ascontiguousarray(np.asarray(v, np.uint32).reshape(-1, 4))
    if a.shape[0] > MAX_SECUREFIELD_VEC_LEN:
        raise ValueError("securefield vector too long")
    return struct.pack("<I", a.shape[0]) + a.astype("<u4").tobytes()


class _Reader:
    def __init__(self, b: bytes):
        self.b, self.pos = b, 0

    def take(self, n: int) -> bytes:
        if self.pos + n > len(self.b):
            raise ValueError("truncated weight cache file")
        out = self.b[self.pos:self.pos + n]
        self.pos += n
        return out

    def u32(self) -> int:
        return struct.unpack("<I", self.take(4))[0]

    def u64(self) -> int:
        return struct.unpack("<Q", self.take(8))[0]

    def sf_vec(self) -> np.ndarray:
        n = self.u32()
        if n > MAX_SECUREFIELD_VEC_LEN:
            raise ValueError(f"securefield vec length {n} exceeds maximum {MAX_SECUREFIELD_VEC_LEN}")
        return np.frombuffer(self.take(16 * n), "<u4").astype(np.uint32).reshape(n, 4)
