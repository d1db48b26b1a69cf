"""Oracle self-consistency (no GPU): the materialised restriction
(backend.rs:127-134) and the fused unpadded one (matmul.rs:470-566) agree, as
the reference's own tests assert (matmul.rs:2156-2218); round polynomials satisfy
p(0)+p(1) = claim."""
import numpy as np
import pytest

import oracle_lib as O
from helpers import int_matrix_m31, log2, next_pow2, random_qm31

SHAPES = [(1, 4, 2), (2, 3, 5), (3, 7, 1), (1, 1, 1), (4, 16, 8), (5, 33, 17), (1, 64, 1), (8, 100, 70)]


@pytest.mark.parametrize("m,k,n", SHAPES)
def test_materialised_equals_fused(m, k, n):
    rng = np.random.default_rng(m * 1000 + k * 10 + n)
    a = int_matrix_m31(m, k, 1)
    b = int_matrix_m31(k, n, 2)
    r_i = random_qm31(log2(next_pow2(m)), rng)
    r_j = random_qm31(log2(next_pow2(n)), rng)
    res = []
    for mode in (0, 1):
        ch = O.new_channel()
        O.lib().orc_ch_mix_u64(O.C.byref(ch), 42)
        res.append((O.reduce_matmul_layer(a, b, r_i, r_j, ch, mode=mode), ch.digest_int()))
    (r0, d0), (r1, d1) = res
    assert d0 == d1
    for key in ("round_polys", "challenges", "final_a", "final_b"):
        assert (r0[key] == r1[key]).all(), key


def qadd(x, y):
    return (x.astype(np.uint64) + y) % O.np.uint64((1 << 31) - 1)


@pytest.mark.parametrize("m,k,n", [(2, 8, 4), (3, 5, 6)])
def test_round_sum_identity(m, k, n):
    """p_r(0) + p_r(1) equals the previous round's p(alpha); final = fa * fb."""
    rng = np.random.default_rng(5)
    a = int_matrix_m31(m, k, 3)
    b = int_matrix_m31(k, n, 4)
    r_i = random_qm31(log2(next_pow2(m)), rng)
    r_j = random_qm31(log2(next_pow2(n)), rng)
    ch = O.new_channel()
    red = O.reduce_matmul_layer(a, b, r_i, r_j, ch)
    P = (1 << 31) - 1

    def add(x, y):
        return ((x.astype(np.int64) + y) % P).astype(np.uint32)

    def mul(x, y):
        out = np.zeros(4, np.uint32)
        O.lib().orc_qm31_mul(np.ascontiguousarray(x, np.uint32), np.ascontiguousarray(y, np.uint32), out)
        return out

    prev = None
    for rp, alpha in zip(red["round_polys"], red["challenges"]):
        c0, c1, c2 = rp[0:4], rp[4:8], rp[8:12]
        s = add(add(c0, c0), add(c1, c2))
        if prev is not None:
            assert (s == prev).all()
        prev = add(add(c0, mul(c1, alpha)), mul(c2, mul(alpha, alpha)))
    assert (prev == mul(red["final_a"], red["final_b"])).all()
