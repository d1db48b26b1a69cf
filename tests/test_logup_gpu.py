"""GPU parity for the LogUp activation layer: bit-exact calldata, transcript and
input evaluation against the oracle, and acceptance by the oracle's verifier."""
import numpy as np
import pytest

import oracle_lib as O
import zkml_b200 as Z
from helpers import int_matrix_m31, log2, next_pow2, random_qm31, uniform_m31

pytestmark = pytest.mark.gpu

CASES = [(1, 8, 5), (2, 3, 5), (1, 1536, 5), (4, 64, 2), (3, 5, 4), (8, 32, 1), (16, 100, 3), (64, 13824, 5)]


@pytest.mark.parametrize("rows,cols,tag", CASES, ids=lambda x: str(x))
def test_activation_logup_matches_oracle(rows, cols, tag):
    x = int_matrix_m31(rows, cols, 17, bound=60000)
    rng = np.random.default_rng(rows + cols + tag)
    nv = log2(next_pow2(rows)) + log2(next_pow2(cols))
    point = random_qm31(nv, rng)
    value = random_qm31(1, rng)[0]
    och = O.new_channel()
    O.lib().orc_ch_mix_u64(O.C.byref(och), 99)
    rc, raw, ie = O.reduce_activation_logup(x, tag, point, value, och)
    assert rc == 0
    zch = Z.PoseidonChannel()
    zch.mix_u64(99)
    proof, claim = Z.reduce_activation_layer(Z.GKRClaim(point, value), Z.M31Matrix.from_numpy(x), tag, zch)
    assert proof.calldata == [O.felt_int(raw[4 * i:4 * i + 4]) for i in range(raw.size // 4)]
    assert (proof.input_eval == ie).all() and (claim.value == ie).all()
    assert zch.digest() == och.digest_int()
    vch = O.new_channel()
    O.lib().orc_ch_mix_u64(O.C.byref(vch), 99)
    ok, _ = O.verify_activation_logup(proof.raw, point, value, vch)
    assert ok and vch.digest_int() == zch.digest()


def test_activation_full_range_inputs():
    x = uniform_m31(4 * 256, 5).reshape(4, 256)
    rng = np.random.default_rng(1)
    point = random_qm31(10, rng)
    value = random_qm31(1, rng)[0]
    rc, raw, ie = O.reduce_activation_logup(x, 5, point, value, O.new_channel())
    proof, _ = Z.reduce_activation_layer(Z.GKRClaim(point, value), Z.M31Matrix.from_numpy(x), 5, Z.PoseidonChannel())
    assert rc == 0 and (proof.raw == raw).all()


def test_activation_rejects_bad_point():
    x = int_matrix_m31(2, 4, 1)
    with pytest.raises(Z.InvalidArgument):
        Z.reduce_activation_layer(Z.GKRClaim(np.zeros((2, 4), np.uint32), np.zeros(4, np.uint32)),
                                  Z.M31Matrix.from_numpy(x), 5, Z.PoseidonChannel())
