"""Product host crypto (felt252 / Hades / channel in libzkml_b200.so) against the
oracle and the reference's known answers.  These functions run on the host, so
they are checked without a GPU."""
import json
import random
from pathlib import Path

import numpy as np
import pytest

import oracle_lib as O
import zkml_b200 as Z

GOLD = json.loads((Path(__file__).parent / "golden" / "reference_vectors.json").read_text())
rng = random.Random(1234)


def rand_felt():
    return rng.randrange(Z.STARK_P)


@pytest.mark.parametrize("kat", GOLD["poseidon_kats"], ids=lambda k: k["op"])
def test_product_poseidon_kats(kat):
    xs = [int(x, 16) for x in kat["inputs"]]
    got = Z.poseidon_hash(*xs) if kat["op"] == "poseidon_hash" else Z.poseidon_hash_many(xs)
    assert got == int(kat["expect"], 16)


def test_hades_compressed_matches_raw_oracle():
    for _ in range(50):
        st = [rand_felt() for _ in range(3)]
        ours = Z.hades_permutation(st)
        ref = np.concatenate([O.felt(x) for x in st])
        O.lib().orc_hades(ref)
        assert ours == [O.felt_int(ref[4 * i:4 * i + 4]) for i in range(3)]


def test_hades_edge_values():
    for st in ([0, 0, 0], [Z.STARK_P - 1] * 3, [1, Z.STARK_P - 1, 0]):
        ref = np.concatenate([O.felt(x) for x in st])
        O.lib().orc_hades(ref)
        assert Z.hades_permutation(st) == [O.felt_int(ref[4 * i:4 * i + 4]) for i in range(3)]


@pytest.mark.parametrize("n", [0, 1, 2, 3, 4, 7, 14])
def test_hash_many_matches_oracle(n):
    xs = [rand_felt() for _ in range(n)]
    assert Z.poseidon_hash_many(xs) == O.poseidon_hash_many(xs)


def test_securefield_to_felt():
    for v in ([0, 0, 0, 0], [1, 2, 3, 4], [Z.M31_P - 1, 17, 1234567, Z.M31_P - 2]):
        arr = np.array(v, np.uint32)
        out = np.zeros(4, np.uint64)
        O.lib().orc_securefield_to_felt(arr, out)
        assert Z.securefield_to_felt(arr) == O.felt_int(out)


def test_channel_transcript_matches_oracle():
    """A random sequence of every channel operation, product vs oracle."""
    zc = Z.PoseidonChannel()
    oc = O.new_channel()
    r = np.random.default_rng(7)
    for step in range(60):
        op = step % 7
        if op == 0:
            v = int(r.integers(0, 2**63))
            zc.mix_u64(v)
            O.lib().orc_ch_mix_u64(O.C.byref(oc), v)
        elif op == 1:
            f = rand_felt()
            zc.mix_felt(f)
            O.lib().orc_ch_mix_felt(O.C.byref(oc), O.felt(f))
        elif op == 2:
            a = zc.draw_qm31()
            b = np.zeros(4, np.uint32)
            O.lib().orc_ch_draw_qm31(O.C.byref(oc), b)
            assert (a == b).all()
            assert (a < Z.M31_P).all()
        elif op == 3:
            c = r.integers(0, Z.M31_P, 12, dtype=np.uint32)
            zc.mix_poly_coeffs(c[0:4], c[4:8], c[8:12])
            O.lib().orc_ch_mix_poly_coeffs(O.C.byref(oc), c)
        elif op == 4:
            c = r.integers(0, Z.M31_P, 16, dtype=np.uint32)
            zc.mix_poly_coeffs_deg3(c[0:4], c[4:8], c[8:12], c[12:16])
            O.lib().orc_ch_mix_poly_coeffs_deg3(O.C.byref(oc), c)
        elif op == 5:
            n = int(r.integers(1, 6))
            q = r.integers(0, Z.M31_P, (n, 4), dtype=np.uint32)
            zc.mix_felts(q)
            O.lib().orc_ch_mix_felts(O.C.byref(oc), q.reshape(-1), n)
        else:
            a = zc.draw_felt252()
            b = np.zeros(4, np.uint64)
            O.lib().orc_ch_draw_felt(O.C.byref(oc), b)
            assert a == O.felt_int(b)
        assert zc.digest() == oc.digest_int()
        assert zc.n_draws() == oc.n_draws


def test_mix_felts_js_reference_vector():
    # poseidon_channel.rs:1619-1637: mix_felts([QM31(1,2,3,4)]) from the zero state
    ch = Z.PoseidonChannel()
    ch.mix_felts([[1, 2, 3, 4]])
    assert ch.digest() == int(GOLD["poseidon_kats"][0]["expect"], 16)


def test_draw_qm31_reduces_2_31_minus_1():
    # A remainder of exactly 2^31 - 1 maps to 0 (BaseField::reduce); exercise many draws.
    ch = Z.PoseidonChannel()
    for _ in range(200):
        assert (ch.draw_qm31() < Z.M31_P).all()


def test_io_commitment_matches_oracle():
    inp = np.array([[1, 2, 3, 4]], np.uint32)
    out = np.array([[50, 60]], np.uint32)
    ref = np.zeros(4, np.uint64)
    O.lib().orc_io_commitment(inp.reshape(-1), 1, 4, out.reshape(-1), 1, 2, ref)
    assert Z.io_commitment(inp, out) == O.felt_int(ref)
    assert Z.io_commitment(inp, out) == int(GOLD["sp3_matmul_only"]["io_commitment"], 16)


@pytest.mark.parametrize("tag", [1, 2, 3, 4, 5])
def test_activation_tables_match_oracle(tag):
    lg = O.lib().orc_activation_table_log_size(tag)
    ref = np.zeros(1 << lg, np.uint32)
    O.lib().orc_activation_table(tag, lg, ref)
    assert (Z.activation_table(tag) == ref).all()


def test_montgomery_multiply_and_cube_edges():
    """The x86 Montgomery multiply and cube (felt252_x86.S) against big-integer arithmetic, on
    inputs up to 4p (5p for the cube: the lazy-reduction ranges) and on products whose low 192 bits are zero
    (the reduction's no-carry path)."""
    import ctypes as C
    import random
    p = Z.STARK_P
    R = 1 << 256
    rinv = pow(R, -1, p)
    L = Z.lib()
    try:
        flags = open("/proc/cpuinfo").read()
    except OSError:
        flags = ""
    if not hasattr(L, "zk_felt_mont_mul_adx") or " adx" not in flags or " bmi2" not in flags:
        pytest.skip("no x86 ADX / BMI2 multiply on this host")
    u64x4 = C.c_uint64 * 4

    def limbs(x):
        return u64x4(*[(x >> (64 * i)) & (2**64 - 1) for i in range(4)])

    def val(a):
        return sum(int(a[i]) << (64 * i) for i in range(4))

    rng = random.Random(7)
    cases = [(0, 0), (1, 1), (p - 1, p - 1), (4 * p - 1, 4 * p - 1), (1 << 192, 1 << 64), (1 << 128, 1 << 128),
             (1 << 250, 1 << 6), (p, p), (2 * p + 5, 3 * p + 7)]
    cases += [(rng.randrange(4 * p), rng.randrange(4 * p)) for _ in range(3000)]
    for a, b in cases:
        r = u64x4()
        L.zk_felt_mont_mul_adx(r, limbs(a), limbs(b))
        assert val(r) == a * b * rinv % p
        if a == b or a < 4 * p:
            # the cube is left unreduced, below 1.3 p, for inputs below 5 p
            for x in (a, a + p):
                L.zk_felt_mont_cube_adx(r, limbs(x))
                assert val(r) % p == x * x * x * rinv * rinv % p and val(r) < 13 * p // 10
