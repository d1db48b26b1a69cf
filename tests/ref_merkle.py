"""Loader for oracle/_ref/libref_merkle.so, the reference's own Poseidon-252 Merkle layer kernel
(built by oracle/build_ref_merkle.py), and the inputs it takes: canonical felts as 4
little-endian u64 limbs and the 107 compressed round keys.  Test and benchmark infrastructure.
"""
import ctypes as C
import re
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[1]
SO = ROOT / "oracle" / "_ref" / "libref_merkle.so"
STARK_P = 2**251 + 17 * 2**192 + 1

_lib = None


def available() -> bool:
    return SO.exists()


def lib():
    global _lib
    if _lib is None:
        _lib = C.CDLL(str(SO))
        _lib.ref_merkle_hash_level.argtypes = [C.c_void_p, C.c_void_p, C.c_uint, C.c_void_p, C.c_void_p]
        _lib.ref_merkle_root.argtypes = [C.c_void_p, C.c_ulonglong, C.c_void_p, C.c_void_p, C.c_void_p]
    return _lib


def raw_round_keys():
    """The 91 x 3 Hades round keys, from the product's generated table (the public poseidon3
    parameter set)."""
    text = (ROOT / "stwo-ml_b200" / "csrc" / "poseidon3_round_keys.inc").read_text()
    vals = []
    for m in re.finditer(r"\{(0x[0-9a-f]+)ULL, (0x[0-9a-f]+)ULL, (0x[0-9a-f]+)ULL, (0x[0-9a-f]+)ULL\}", text):
        vals.append(sum(int(m.group(i + 1), 16) << (64 * i) for i in range(4)))
    assert len(vals) == 273
    return [vals[3 * r:3 * r + 3] for r in range(91)]


def compressed_round_keys():
    """The 107 keys of the optimised schedule (cuda_executor.rs:5174-5222): the first four full
    rounds' keys, one key per partial round with the other two pushed through the MDS mix,
    the keys of the first of the last full rounds with the carried state added, then the
    remaining three full rounds' keys."""
    p = STARK_P
    raw = raw_round_keys()
    comp = [k for r in raw[:4] for k in r]
    st = [0, 0, 0]
    idx = 4
    for _ in range(83):
        st = [(st[i] + raw[idx][i]) % p for i in range(3)]
        comp.append(st[2])
        st[2] = 0
        t = (st[0] + st[1] + st[2]) % p
        st = [(t + 2 * st[0]) % p, (t - 2 * st[1]) % p, (t - 3 * st[2]) % p]
        idx += 1
    st = [(st[i] + raw[idx][i]) % p for i in range(3)]
    comp.extend(st)
    for r in raw[idx + 1:]:
        comp.extend(r)
    assert len(comp) == 107
    return comp


def limbs(values) -> np.ndarray:
    """Canonical integers -> (len, 4) little-endian u64 limbs."""
    out = np.zeros((len(values), 4), np.uint64)
    for i, v in enumerate(values):
        for j in range(4):
            out[i, j] = (v >> (64 * j)) & (2**64 - 1)
    return out


def leaf_felts(qm31: np.ndarray) -> np.ndarray:
    """securefield_to_felt of QM31 leaves (2^124 | a << 93 | b << 62 | c << 31 | d) as limbs."""
    q = np.asarray(qm31, np.uint64).reshape(-1, 4)
    a, b, c, d = q[:, 0], q[:, 1], q[:, 2], q[:, 3]
    lo = d | (c << np.uint64(31)) | (b << np.uint64(62))
    hi = (b >> np.uint64(2)) | (a << np.uint64(29)) | np.uint64(1 << 60)
    out = np.zeros((len(q), 4), np.uint64)
    out[:, 0], out[:, 1] = lo, hi
    return out
