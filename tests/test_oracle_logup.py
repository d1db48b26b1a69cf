"""Oracle LogUp activation layer (no GPU): prove -> verifier replay round trip,
tamper rejection, and the activation tables' defining properties."""
import numpy as np
import pytest

import oracle_lib as O
from helpers import int_matrix_m31, log2, next_pow2, random_qm31

P = (1 << 31) - 1


def table(tag):
    lg = O.lib().orc_activation_table_log_size(tag)
    t = np.zeros(1 << lg, np.uint32)
    assert O.lib().orc_activation_table(tag, lg, t) == 0
    return t


def test_tables_basic_values():
    relu = table(1)
    assert (relu[:5] == np.arange(5)).all()
    silu = table(5)
    assert silu[0] == 0 and silu[65536 // 2] > 0  # silu(0.5) ~ 0.311 -> ~20385
    assert abs(int(silu[65536 // 2]) - round(0.5 / (1 + np.exp(-0.5)) * 65536)) <= 1
    sm = table(4)
    assert sm[0] == 65536 and sm[65536] == 131072
    sig = table(3)
    assert sig[0] == 32768 and sig[5] == 65536


def mk_claim(rows, cols, seed):
    rng = np.random.default_rng(seed)
    nv = log2(next_pow2(rows)) + log2(next_pow2(cols))
    return random_qm31(nv, rng), random_qm31(1, rng)[0]


@pytest.mark.parametrize("rows,cols,tag", [(1, 8, 5), (2, 3, 5), (1, 1536, 5), (4, 64, 2), (3, 5, 4), (8, 32, 1)])
def test_logup_prove_verify_roundtrip(rows, cols, tag):
    x = int_matrix_m31(rows, cols, 7, bound=40000)
    point, value = mk_claim(rows, cols, rows * 31 + cols)
    ch = O.new_channel()
    rc, raw, ie = O.reduce_activation_logup(x, tag, point, value, ch)
    assert rc == 0
    vch = O.new_channel()
    ok, ie2 = O.verify_activation_logup(raw, point, value, vch)
    assert ok and (ie == ie2).all()
    assert vch.digest_int() == ch.digest_int()
    bad = raw.copy()
    bad[4 * 12] ^= 1  # claimed sum word
    assert not O.verify_activation_logup(bad, point, value, O.new_channel())[0]
