"""Packed host -> device upload of B (csrc/h2d_pack.cu) inside zkml_reduce_matmul_layer.

A host B whose words are the M31 images of signed bytes crosses PCIe as one byte per word, in
chunks of 2^18 words; a chunk with any other word goes over unchanged.  The proof must be the
oracle's, bit for bit, whichever way each chunk travelled, and the bytes the context counts must
show which way that was.  ZKML_PACK_MIN=1 makes every host B take the packed path here (the
default threshold is 2^22 words; the full config-2 B of tests/test_matmul_gpu.py takes it by
default).
"""
import numpy as np
import pytest

import oracle_lib as O
import zkml_b200 as Z
from helpers import M31_P, int_matrix_m31, log2, next_pow2, random_qm31

pytestmark = pytest.mark.gpu

CHUNK = 1 << 18


def prove(a, b, seed):
    m, k = a.shape
    n = b.shape[1]
    rng = np.random.default_rng(seed)
    r_i = random_qm31(log2(next_pow2(m)), rng)
    r_j = random_qm31(log2(next_pow2(n)), rng)
    be = Z.GpuBackend(0)
    before = be.ctx.h2d_bytes()
    got = be.reduce_matmul_layer(Z.M31Matrix.from_numpy(a), Z.M31Matrix.from_numpy(b), r_i, r_j, next_pow2(k),
                                 Z.PoseidonChannel())
    return got, be.ctx.h2d_bytes() - before, (r_i, r_j)


def oracle(a, b, pts):
    return O.reduce_matmul_layer(a, b, pts[0], pts[1], O.new_channel(), mode=1)


def same(got, ref):
    for r, rp in enumerate(got.round_polys):
        assert (np.concatenate([rp.c0, rp.c1, rp.c2]) == ref["round_polys"][r]).all(), f"round {r}"
    assert (got.final_a_eval == ref["final_a"]).all() and (got.final_b_eval == ref["final_b"]).all()


def chunks(b):
    return -(-b.size // CHUNK)  # one packed/raw flag byte per chunk also crosses


def byte_matrix(k, n, seed):
    b = int_matrix_m31(k, n, seed, bound=128)  # [-128, 128]: 128 is out of range, clamp it
    b[b == 128] = 127
    flat = b.reshape(-1)
    flat[:4] = [0, 127, M31_P - 128, M31_P]  # extremes, and p itself (the zero element)
    return b


@pytest.fixture
def pack_small(monkeypatch):
    monkeypatch.setenv("ZKML_PACK_MIN", "1")
    monkeypatch.delenv("ZKML_PACK_H2D", raising=False)


def test_packed_chunks_match_oracle(pack_small):
    a = int_matrix_m31(4, 1100, 31)
    b = byte_matrix(1100, 1000, 32)  # 1.1 M words: five chunks, the last ragged
    got, h2d, pts = prove(a, b, 5)
    same(got, oracle(a, b, pts))
    assert h2d == a.size * 4 + b.size + chunks(b)  # A as words, every chunk of B as bytes


def test_raw_chunk_beside_packed_one(pack_small):
    a = int_matrix_m31(4, 1100, 33)
    b = byte_matrix(1100, 1000, 34)
    b.reshape(-1)[CHUNK + 5] = 1000  # not a signed byte: the second chunk goes as words
    got, h2d, pts = prove(a, b, 6)
    same(got, oracle(a, b, pts))
    assert h2d == a.size * 4 + (b.size - CHUNK) + CHUNK * 4 + chunks(b)


def test_packing_off_gives_the_same_proof(monkeypatch):
    a = int_matrix_m31(8, 300, 35)
    b = byte_matrix(300, 260, 36)
    monkeypatch.setenv("ZKML_PACK_MIN", "1")
    packed, h_on, pts = prove(a, b, 7)
    monkeypatch.setenv("ZKML_PACK_H2D", "0")
    plain, h_off, _ = prove(a, b, 7)
    same(packed, oracle(a, b, pts))
    for x, y in zip(packed.round_polys, plain.round_polys):
        assert (x.c0 == y.c0).all() and (x.c1 == y.c1).all() and (x.c2 == y.c2).all()
    assert h_on == a.size * 4 + b.size + chunks(b) and h_off == (a.size + b.size) * 4


def test_word_with_bit31_still_rejected(pack_small):
    a = int_matrix_m31(2, 64, 37)
    b = byte_matrix(64, 40, 38)
    b[3, 7] = 0x80000005
    with pytest.raises(Z.InvalidArgument):
        prove(a, b, 8)
    # the context stays usable
    b[3, 7] = 1
    got, _, pts = prove(a, b, 9)
    same(got, oracle(a, b, pts))
