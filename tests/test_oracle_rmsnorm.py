"""Oracle RMSNorm layer (no GPU): the rsqrt table's defining values, prove ->
verifier replay round trip with identical transcripts, tamper rejection, and a
direct recomputation of the per-row rms^2 values the record carries."""
import numpy as np
import pytest

import oracle_lib as O
from helpers import int_matrix_m31, log2, next_pow2, random_qm31

P = (1 << 31) - 1


def test_rsqrt_table_values():
    t = O.rsqrt_table(16)
    assert t[0] == 65535 and t[1] == 65536 and t[4] == 32768 and t[3] == 65536
    import math
    for x in [2, 5, 99, 1000, 65535, 12345]:
        assert t[x] == 65536 // math.isqrt(x)


def honest_claim(x, dim, seed, gamma=None):
    rows, cols = x.shape
    nv = log2(next_pow2(rows)) + log2(next_pow2(cols))
    rng = np.random.default_rng(seed)
    point = random_qm31(nv, rng)
    rc, raw, _ = O.reduce_rmsnorm(x, dim, point, np.zeros(4, np.uint32), O.new_channel(), gamma=gamma)
    assert rc == 0
    return point, O.rmsnorm_output_eval(raw)


def row_rms_expected(x, dim):
    rows, cols = x.shape
    pr, pc = next_pow2(rows), next_pow2(cols)
    na = min(dim, pc)
    xp = np.zeros((pr, pc), np.int64)
    xp[:rows, :cols] = x
    inv = pow(na, P - 2, P)
    out = []
    for i in range(pr):
        s = 0
        for j in range(na):
            s = (s + int(xp[i, j]) * int(xp[i, j])) % P
        out.append((s * inv % P) & 0xFFFF)
    return out


@pytest.mark.parametrize("rows,cols,gamma", [(1, 8, False), (2, 3, False), (4, 64, True), (3, 5, True),
                                             (8, 32, False), (1, 1536, False)])
def test_rmsnorm_prove_verify_roundtrip(rows, cols, gamma):
    x = int_matrix_m31(rows, cols, 11, bound=300)
    g = (np.arange(cols, dtype=np.uint32) * 37 + 5) % 1000 if gamma else None
    point, value = honest_claim(x, cols, rows * 7 + cols, g)
    ch = O.new_channel()
    O.lib().orc_ch_mix_u64(O.C.byref(ch), 5)
    rc, raw, ie = O.reduce_rmsnorm(x, cols, point, value, ch, gamma=g)
    assert rc == 0
    vch = O.new_channel()
    O.lib().orc_ch_mix_u64(O.C.byref(vch), 5)
    ok, ie2 = O.verify_rmsnorm(raw, cols, point, value, vch)
    assert ok and (ie == ie2).all()
    assert vch.digest_int() == ch.digest_int()
    # the record's per-row rms^2 values
    if next_pow2(rows) > 1:
        tail = [O.felt_int(raw[4 * i:4 * i + 4]) for i in range(raw.size // 4 - next_pow2(rows), raw.size // 4)]
        assert tail == row_rms_expected(x, cols)
    # tampering: a wrong claim value, a flipped round word
    bad_value = value.copy()
    bad_value[0] = (bad_value[0] + 1) % P
    assert not O.verify_rmsnorm(raw, cols, point, bad_value, O.new_channel())[0]
    bad = raw.copy()
    bad[4 * 40] ^= 1
    assert not O.verify_rmsnorm(bad, cols, point, value, O.new_channel())[0]


def test_rmsnorm_skip_rms_sq_changes_record():
    x = int_matrix_m31(2, 8, 3, bound=100)
    point, value = honest_claim(x, 8, 1)
    rc0, raw0, ie0 = O.reduce_rmsnorm(x, 8, point, value, O.new_channel())
    rc1, raw1, ie1 = O.reduce_rmsnorm(x, 8, point, value, O.new_channel(), skip_rms_sq=True)
    assert rc0 == rc1 == 0 and (ie0 == ie1).all()
    assert raw1.size < raw0.size
    # a record without the RMS^2 proof is rejected by the verifier
    assert not O.verify_rmsnorm(raw1, 8, point, value, O.new_channel())[0]
