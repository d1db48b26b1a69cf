"""GPU parity for the piecewise-linear activation reduction (the reference's default
non-ReLU activation proof): bit-exact calldata, next claim and transcript against the
oracle, and acceptance by the oracle's verifier."""
import numpy as np
import pytest

import oracle_lib as O
import zkml_b200 as Z
from helpers import int_matrix_m31, random_qm31, uniform_m31

pytestmark = pytest.mark.gpu

CASES = [(1, 2, 5), (1, 4, 5), (1, 8, 2), (2, 3, 3), (4, 16, 4), (3, 5, 5), (8, 32, 1), (16, 100, 5),
         (64, 1000, 2), (33, 257, 5)]


@pytest.mark.parametrize("rows,cols,tag", CASES, ids=lambda x: str(x))
def test_piecewise_matches_oracle(rows, cols, tag):
    x = uniform_m31(rows * cols, rows * 7 + cols).reshape(rows, cols)
    rng = np.random.default_rng(rows + 3 * cols + tag)
    nv = (rows - 1).bit_length() + (cols - 1).bit_length()
    point, value = random_qm31(nv, rng), random_qm31(1, rng)[0]
    och = O.new_channel()
    O.lib().orc_ch_mix_u64(O.C.byref(och), 21)
    rc, raw, ie, nxt = O.reduce_activation_piecewise(x, tag, point, value, och)
    assert rc == 0
    zch = Z.PoseidonChannel()
    zch.mix_u64(21)
    proof, claim = Z.reduce_activation_layer_piecewise(Z.GKRClaim(point, value), Z.M31Matrix.from_numpy(x), tag, zch)
    assert proof.raw.size == raw.size and (proof.raw == raw).all()
    assert (claim.value == ie).all() and (claim.point == nxt).all()
    assert zch.digest() == och.digest_int()
    vch = O.new_channel()
    O.lib().orc_ch_mix_u64(O.C.byref(vch), 21)
    ok, _ = O.verify_activation_piecewise(proof.raw, point, value, vch)
    assert ok and vch.digest_int() == zch.digest()


def test_piecewise_small_values_and_device_input():
    import torch
    x = int_matrix_m31(16, 64, 4, bound=60000)
    rng = np.random.default_rng(2)
    point, value = random_qm31(10, rng), random_qm31(1, rng)[0]
    rc, raw, ie, nxt = O.reduce_activation_piecewise(x, 5, point, value, O.new_channel())
    xd = torch.from_numpy(x.view(np.int32)).cuda().reshape(-1)
    proof, _ = Z.reduce_activation_layer_piecewise(Z.GKRClaim(point, value), Z.M31Matrix(16, 64, xd), 5,
                                                   Z.PoseidonChannel())
    assert rc == 0 and (proof.raw == raw).all()
