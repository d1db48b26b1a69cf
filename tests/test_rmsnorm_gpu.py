"""GPU parity for the RMSNorm layer reduction: bit-exact calldata, transcript and
input evaluation against the oracle (with and without the affine scale, with the
RMS^2 proof skipped by STWO_SKIP_RMS_SQ_PROOF), and acceptance by the oracle's
verifier on honest claims."""
import numpy as np
import pytest

import oracle_lib as O
import zkml_b200 as Z
from helpers import int_matrix_m31, log2, next_pow2, random_qm31, uniform_m31

pytestmark = pytest.mark.gpu

CASES = [(1, 2, 2, False), (1, 8, 8, False), (2, 3, 3, True), (4, 64, 64, True), (3, 5, 4, False),
         (8, 32, 32, False), (16, 100, 100, True), (1, 1536, 1536, False), (64, 4096, 4096, True),
         (5, 40, 64, False)]


def claim(x, seed):
    rows, cols = x.shape
    nv = log2(next_pow2(rows)) + log2(next_pow2(cols))
    rng = np.random.default_rng(seed)
    return random_qm31(nv, rng), random_qm31(1, rng)[0]


@pytest.mark.parametrize("rows,cols,dim,gamma", CASES, ids=lambda x: str(x))
def test_rmsnorm_matches_oracle(rows, cols, dim, gamma):
    x = int_matrix_m31(rows, cols, 23, bound=400)
    g = ((np.arange(cols, dtype=np.uint64) * 7919 + 3) % 60000).astype(np.uint32) if gamma else None
    point, value = claim(x, rows * 131 + cols)
    och = O.new_channel()
    O.lib().orc_ch_mix_u64(O.C.byref(och), 77)
    rc, raw, ie = O.reduce_rmsnorm(x, dim, point, value, och, gamma=g)
    assert rc == 0
    zch = Z.PoseidonChannel()
    zch.mix_u64(77)
    proof, nxt = Z.reduce_rmsnorm_layer(Z.GKRClaim(point, value), Z.M31Matrix.from_numpy(x), dim, zch, gamma=g)
    assert proof.raw.size == raw.size and (proof.raw == raw).all()
    assert (proof.input_eval == ie).all() and (nxt.value == ie).all()
    assert zch.digest() == och.digest_int()


@pytest.mark.parametrize("rows,cols", [(2, 8), (4, 64), (32, 1024)])
def test_rmsnorm_honest_claim_verifies(rows, cols):
    x = int_matrix_m31(rows, cols, 5, bound=1000)
    point, _ = claim(x, 3)
    p0, _ = Z.reduce_rmsnorm_layer(Z.GKRClaim(point, np.zeros(4, np.uint32)), Z.M31Matrix.from_numpy(x), cols,
                                   Z.PoseidonChannel())
    value = p0.output_eval
    zch = Z.PoseidonChannel()
    proof, _ = Z.reduce_rmsnorm_layer(Z.GKRClaim(point, value), Z.M31Matrix.from_numpy(x), cols, zch)
    vch = O.new_channel()
    ok, ie = O.verify_rmsnorm(proof.raw, cols, point, value, vch)
    assert ok and (ie == proof.input_eval).all() and vch.digest_int() == zch.digest()


def test_rmsnorm_skip_rms_sq(monkeypatch):
    x = int_matrix_m31(4, 16, 9, bound=200)
    point, value = claim(x, 4)
    rc, raw, ie = O.reduce_rmsnorm(x, 16, point, value, O.new_channel(), skip_rms_sq=True)
    monkeypatch.setenv("STWO_SKIP_RMS_SQ_PROOF", "1")
    proof, _ = Z.reduce_rmsnorm_layer(Z.GKRClaim(point, value), Z.M31Matrix.from_numpy(x), 16, Z.PoseidonChannel())
    assert rc == 0 and (proof.raw == raw).all()


def test_rmsnorm_full_range_and_device_input():
    import torch
    x = uniform_m31(8 * 128, 12).reshape(8, 128)
    point, value = claim(x, 6)
    rc, raw, ie = O.reduce_rmsnorm(x, 128, point, value, O.new_channel())
    xd = torch.from_numpy(x.view(np.int32)).cuda()
    proof, _ = Z.reduce_rmsnorm_layer(Z.GKRClaim(point, value), Z.M31Matrix(8, 128, xd.reshape(-1)), 128, Z.PoseidonChannel())
    assert rc == 0 and (proof.raw == raw).all()


def test_rmsnorm_rejects_bad_point():
    x = int_matrix_m31(2, 4, 1)
    with pytest.raises(Z.InvalidArgument):
        Z.reduce_rmsnorm_layer(Z.GKRClaim(np.zeros((2, 4), np.uint32), np.zeros(4, np.uint32)),
                               Z.M31Matrix.from_numpy(x), 4, Z.PoseidonChannel())
