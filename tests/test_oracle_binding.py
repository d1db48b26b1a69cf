"""Oracle aggregated weight binding (no GPU): honest claims prove and verify with
identical transcripts, for equal and mixed matrix sizes, one claim, and group-offset
matrix indices; a wrong claimed value or commitment is rejected."""
import numpy as np
import pytest

import oracle_lib as O
from helpers import int_matrix_m31, random_qm31


def honest_specs(shapes, seed, index_base=0):
    rng = np.random.default_rng(seed)
    specs = []
    for i, (r, c) in enumerate(shapes):
        w = int_matrix_m31(r, c, seed * 10 + i, bound=1000)
        mle = O.mle_col_major(w)
        nv = mle.shape[0].bit_length() - 1
        pt = random_qm31(nv, rng)
        specs.append((w, index_base + i, pt, O.evaluate_mle(mle, pt), O.weight_commitment(w)))
    return specs


CASES = [([(4, 8), (8, 4)], 0), ([(4, 8), (2, 2), (8, 16)], 0), ([(16, 8)], 0), ([(3, 5), (4, 4), (2, 7), (5, 3)], 4),
         ([(2, 4), (4, 2), (1, 8)], 8)]


@pytest.mark.parametrize("shapes,base", CASES, ids=lambda x: str(x))
def test_binding_roundtrip(shapes, base):
    specs = honest_specs(shapes, len(shapes) + base)
    ch = O.new_channel()
    O.lib().orc_ch_mix_u64(O.C.byref(ch), 3)
    rc, raw = O.prove_aggregated_binding(specs, ch, n_queries=4)
    assert rc == 0
    vch = O.new_channel()
    O.lib().orc_ch_mix_u64(O.C.byref(vch), 3)
    assert O.verify_aggregated_binding(specs, raw, vch, n_queries=4)
    assert vch.digest_int() == ch.digest_int()


def test_binding_rejects_wrong_value_and_commitment():
    specs = honest_specs([(4, 8), (2, 2), (8, 16)], 7)
    bad = list(specs)
    w, idx, pt, val, com = bad[1]
    val = val.copy()
    val[0] = (val[0] + 1) % ((1 << 31) - 1)
    bad[1] = (w, idx, pt, val, com)
    rc, raw = O.prove_aggregated_binding(bad, O.new_channel(), n_queries=4)
    assert rc == 0
    assert not O.verify_aggregated_binding(bad, raw, O.new_channel(), n_queries=4)
    bad = list(specs)
    w, idx, pt, val, com = bad[0]
    com = com.copy()
    com[0] ^= 1
    bad[0] = (w, idx, pt, val, com)
    rc, raw = O.prove_aggregated_binding(bad, O.new_channel(), n_queries=4)
    assert rc == 4
