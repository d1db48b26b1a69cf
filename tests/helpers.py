"""Seeded synthetic inputs shared by the tests and bench.py.

SplitMix64 seeded with the XOR of the four little-endian u64 words of a fixed
32-byte seed; int8 (or int16) values embedded in M31 as x >= 0 ? x : p + x
(the reference's quantize_value, engine/src/gadgets/quantize.rs:105-110).
"""
import numpy as np

M31_P = (1 << 31) - 1
SEED32 = bytes(range(32))


def seed_u64(seed: bytes = SEED32) -> int:
    s = 0
    for i in range(4):
        s ^= int.from_bytes(seed[8 * i:8 * i + 8], "little")
    return s


def splitmix64(state: int, n: int) -> np.ndarray:
    """n outputs of SplitMix64 from `state` (vectorised)."""
    idx = np.arange(1, n + 1, dtype=np.uint64)
    with np.errstate(over="ignore"):
        z = np.uint64(state) + idx * np.uint64(0x9E3779B97F4A7C15)
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        z = z ^ (z >> np.uint64(31))
    return z


def int_matrix_m31(rows: int, cols: int, stream: int, bound: int = 127) -> np.ndarray:
    """Uniform integers in [-bound, bound] embedded in M31, row-major uint32."""
    z = splitmix64(seed_u64() ^ (stream * 0xD1B54A32D192ED03 & (2**64 - 1)), rows * cols)
    v = (z % np.uint64(2 * bound + 1)).astype(np.int64) - bound
    v = np.where(v >= 0, v, M31_P + v).astype(np.uint32)
    return v.reshape(rows, cols)


def uniform_m31(n: int, stream: int) -> np.ndarray:
    z = splitmix64(seed_u64() ^ (stream * 0xD1B54A32D192ED03 & (2**64 - 1)), n)
    return (z % np.uint64(M31_P)).astype(np.uint32)


def random_qm31(n: int, rng: np.random.Generator) -> np.ndarray:
    return rng.integers(0, M31_P, (n, 4), dtype=np.uint32)


def next_pow2(x: int) -> int:
    return 1 << max(0, (x - 1).bit_length())


def log2(x: int) -> int:
    return x.bit_length() - 1
