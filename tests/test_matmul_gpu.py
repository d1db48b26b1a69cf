"""GPU parity: zkml_reduce_matmul_layer (CUDA, through the C ABI) against the
CPU oracle, bit for bit, on the same seeded inputs."""
import numpy as np
import pytest

import oracle_lib as O
import zkml_b200 as Z
from helpers import int_matrix_m31, log2, next_pow2, random_qm31, uniform_m31

pytestmark = pytest.mark.gpu

SHAPES = [
    (1, 4, 2),        # the sp3 golden shape
    (1, 1, 1),        # pk = 1: zero rounds
    (1, 2, 1),        # product sumcheck, one round
    (2, 3, 5),        # all dimensions padded
    (3, 7, 1),        # n = 1 column
    (1, 64, 1),       # 1 x k . k x 1: base-field first round
    (1, 1 << 12, 1),
    (4, 16, 8),
    (5, 33, 17),      # odd n: scalar-load restriction path
    (8, 100, 70),
    (1, 576, 1536),   # BASELINE config 1 (SmolLM2 up-proj)
    (64, 640, 1000),
    (16, 1000, 4099),
]


def run_pair(a, b, seed):
    m, k = a.shape
    n = b.shape[1]
    rng = np.random.default_rng(seed)
    r_i = random_qm31(log2(next_pow2(m)), rng)
    r_j = random_qm31(log2(next_pow2(n)), rng)
    pk = next_pow2(k)
    och = O.new_channel()
    O.lib().orc_ch_mix_u64(O.C.byref(och), seed)
    ref = O.reduce_matmul_layer(a, b, r_i, r_j, och, mode=1)
    zch = Z.PoseidonChannel()
    zch.mix_u64(seed)
    got = Z.GpuBackend().reduce_matmul_layer(Z.M31Matrix.from_numpy(a), Z.M31Matrix.from_numpy(b), r_i, r_j, pk, zch)
    return ref, och, got, zch


def assert_same(ref, och, got, zch):
    log_k = len(ref["round_polys"])
    assert len(got.round_polys) == log_k
    for r in range(log_k):
        rp = np.concatenate([got.round_polys[r].c0, got.round_polys[r].c1, got.round_polys[r].c2])
        assert (rp == ref["round_polys"][r]).all(), f"round {r}"
    assert (got.challenges == ref["challenges"]).all()
    assert (got.final_a_eval == ref["final_a"]).all()
    assert (got.final_b_eval == ref["final_b"]).all()
    assert zch.digest() == och.digest_int()
    assert zch.n_draws() == och.n_draws


@pytest.mark.parametrize("m,k,n", SHAPES, ids=lambda x: str(x))
def test_reduce_matmul_layer_matches_oracle(m, k, n):
    a = int_matrix_m31(m, k, 11)
    b = int_matrix_m31(k, n, 12)
    assert_same(*run_pair(a, b, m * 7 + k * 3 + n))


def test_full_range_m31_values():
    # uniform M31 (not int8) exercises the lazy-reduction bounds
    a = uniform_m31(8 * 300, 21).reshape(8, 300)
    b = uniform_m31(300 * 260, 22).reshape(300, 260)
    assert_same(*run_pair(a, b, 3))


def test_extreme_values():
    P = Z.M31_P
    a = np.full((4, 130), P - 1, np.uint32)
    b = np.full((130, 200), P - 1, np.uint32)
    assert_same(*run_pair(a, b, 4))
    a[:] = P  # the non-canonical zero 2^31 - 1 is accepted and treated as 0
    ref_a = np.zeros_like(a)
    r1 = run_pair(ref_a, b, 5)
    r2 = run_pair(a, b, 5)
    assert (r1[2].final_b_eval == r2[2].final_b_eval).all()
    assert (r1[2].final_a_eval == r2[2].final_a_eval).all()


def test_rejects_values_above_2_31():
    a = int_matrix_m31(2, 8, 1)
    b = int_matrix_m31(8, 4, 2)
    b[3, 1] = 0x80000005
    with pytest.raises(Z.InvalidArgument):
        run_pair(a, b, 1)
    # the context stays usable
    assert_same(*run_pair(a, int_matrix_m31(8, 4, 2), 1))


def test_rejects_bad_shapes():
    be = Z.GpuBackend()
    ch = Z.PoseidonChannel()
    a = Z.M31Matrix.from_numpy(int_matrix_m31(2, 8, 1))
    b = Z.M31Matrix.from_numpy(int_matrix_m31(7, 4, 2))
    with pytest.raises(Z.InvalidArgument):
        be.reduce_matmul_layer(a, b, np.zeros((1, 4), np.uint32), np.zeros((2, 4), np.uint32), 8, ch)
    b = Z.M31Matrix.from_numpy(int_matrix_m31(8, 4, 2))
    with pytest.raises(Z.InvalidArgument):  # wrong r_j length
        be.reduce_matmul_layer(a, b, np.zeros((1, 4), np.uint32), np.zeros((3, 4), np.uint32), 8, ch)


def test_device_resident_inputs_match_host():
    import torch
    a = int_matrix_m31(16, 512, 31)
    b = int_matrix_m31(512, 300, 32)
    ref, och, got, zch = run_pair(a, b, 9)
    rng = np.random.default_rng(9)
    r_i = random_qm31(4, rng)
    r_j = random_qm31(9, rng)
    ta = torch.from_numpy(a.view(np.int32)).cuda()
    tb = torch.from_numpy(b.view(np.int32)).cuda()
    zc = Z.PoseidonChannel()
    zc.mix_u64(9)
    got2 = Z.GpuBackend().reduce_matmul_layer(Z.M31Matrix(16, 512, ta), Z.M31Matrix(512, 300, tb), r_i, r_j, 512, zc)
    assert_same(ref, och, got2, zc)


def test_transcript_wrapper_matches_oracle():
    m, k, n = 6, 40, 24
    a = int_matrix_m31(m, k, 41)
    b = int_matrix_m31(k, n, 42)
    rng = np.random.default_rng(3)
    point = random_qm31(log2(next_pow2(m)) + log2(next_pow2(n)), rng)
    value = random_qm31(1, rng)[0]
    och = O.new_channel()
    rp = np.zeros((6, 12), np.uint32)
    fa = np.zeros(4, np.uint32)
    fb = np.zeros(4, np.uint32)
    nxt = np.zeros((3 + 6, 4), np.uint32)
    rc = O.lib().orc_reduce_matmul_gkr(point.reshape(-1), len(point), value, a.reshape(-1), m, k, b.reshape(-1), n,
                                       O.C.byref(och), rp.reshape(-1), fa, fb, nxt.reshape(-1), 1, 4)
    assert rc == 0
    zch = Z.PoseidonChannel()
    red, claim = Z.reduce_matmul_layer_with_backend(Z.GKRClaim(point, value), Z.M31Matrix.from_numpy(a),
                                                    Z.M31Matrix.from_numpy(b), m, k, n, zch)
    assert zch.digest() == och.digest_int()
    assert (claim.point == nxt).all()
    assert (claim.value == fa).all() and (red.final_b_eval == fb).all()


@pytest.mark.parametrize("n_vars", [0, 1, 5, 12])
def test_evaluate_and_restrict_mle(n_vars):
    rng = np.random.default_rng(n_vars)
    mle = random_qm31(1 << n_vars, rng)
    pt = random_qm31(n_vars, rng)
    out = np.zeros(4, np.uint32)
    O.lib().orc_evaluate_mle(mle.reshape(-1), n_vars, pt.reshape(-1) if n_vars else np.zeros(4, np.uint32), out)
    be = Z.GpuBackend()
    assert (be.evaluate_mle_at_point(mle, pt) == out).all()
    for n_assign in range(0, n_vars + 1, 3):
        ref = np.zeros(((1 << n_vars) >> n_assign, 4), np.uint32)
        O.lib().orc_restrict_mle(mle.reshape(-1), 1 << n_vars,
                                 pt[:n_assign].reshape(-1) if n_assign else np.zeros(4, np.uint32), n_assign,
                                 ref.reshape(-1))
        assert (be.restrict_mle(mle, pt[:n_assign]) == ref).all()


def test_c2_full_shape_matches_oracle():
    """64 x 5120 . 5120 x 13824 (padded 64 x 8192, 8192 x 16384)."""
    a = int_matrix_m31(64, 5120, 1)
    b = int_matrix_m31(5120, 13824, 2)
    assert_same(*run_pair(a, b, 2024))


def test_repeated_calls_are_deterministic():
    a = int_matrix_m31(8, 300, 5)
    b = int_matrix_m31(300, 130, 6)
    r1 = run_pair(a, b, 77)
    r2 = run_pair(a, b, 77)
    assert (r1[2].final_b_eval == r2[2].final_b_eval).all()
    assert r1[3].digest() == r2[3].digest()
