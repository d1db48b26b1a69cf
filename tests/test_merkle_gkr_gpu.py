"""GPU parity for the Poseidon Merkle commitment, the MLE opening proof and the
single-layer GKR proof, against the oracle and the reference's golden artifact."""
import json
from pathlib import Path

import numpy as np
import pytest

import oracle_lib as O
import zkml_b200 as Z
from helpers import int_matrix_m31, random_qm31

pytestmark = pytest.mark.gpu
GOLD = json.loads((Path(__file__).parent / "golden" / "reference_vectors.json").read_text())


@pytest.mark.parametrize("n", [1, 2, 3, 5, 8, 255, 256, 1000, 1 << 14])
def test_commit_root_matches_oracle(n):
    rng = np.random.default_rng(n)
    ev = random_qm31(n, rng)
    assert Z.commit_mle_root(ev) == O.merkle_root_qm31(ev)


def oracle_opening(ev, pt, nq, seed):
    och = O.new_channel()
    O.lib().orc_ch_mix_u64(O.C.byref(och), seed)
    n_vars = len(pt)
    cap = 1 << 16
    buf = np.zeros(4 * cap, np.uint64)
    com = np.zeros(4, np.uint64)
    ln = O.C.c_size_t(0)
    rc = O.lib().orc_prove_mle_opening(ev.reshape(-1), n_vars, pt.reshape(-1) if n_vars else np.zeros(4, np.uint32),
                                       O.C.byref(och), nq, com, buf, cap, O.C.byref(ln), 4)
    assert rc == 0
    return O.felt_int(com), [O.felt_int(buf[4 * i:4 * i + 4]) for i in range(ln.value)], och


@pytest.mark.parametrize("n_vars,nq", [(0, 10), (1, 10), (2, 10), (3, 10), (6, 2), (8, 10), (12, 20), (16, 10)])
def test_mle_opening_matches_oracle(n_vars, nq):
    rng = np.random.default_rng(100 + n_vars)
    ev = random_qm31(1 << n_vars, rng)
    pt = random_qm31(n_vars, rng)
    com, cd, och = oracle_opening(ev, pt, nq, n_vars)
    zch = Z.PoseidonChannel()
    zch.mix_u64(n_vars)
    got = Z.prove_mle_opening(ev, pt, zch, n_queries=nq)
    assert got.commitment == com
    assert got.calldata == cd
    assert zch.digest() == och.digest_int()
    # the oracle's verifier (restating mle_opening.rs:1918-2029) accepts it
    vch = O.new_channel()
    O.lib().orc_ch_mix_u64(O.C.byref(vch), n_vars)
    raw = np.concatenate([O.felt(x) for x in got.calldata]).astype(np.uint64)
    fin = np.zeros(4, np.uint32)
    ok = O.lib().orc_verify_mle_opening(O.felt(got.commitment), raw, len(got.calldata),
                                        pt.reshape(-1) if n_vars else np.zeros(4, np.uint32), n_vars,
                                        O.C.byref(vch), nq, fin)
    assert ok and vch.digest_int() == zch.digest()


def test_gkr_matmul_reproduces_sp3_artifact():
    """The B200 prover reproduces engine/tests/artifacts/sp3_matmul_only_proof.json byte for byte."""
    g = GOLD["sp3_matmul_only"]
    inp = Z.M31Matrix.from_numpy(np.array([g["input"]], np.uint32))
    w = Z.M31Matrix.from_numpy(np.array(g["weight"], np.uint32))
    proof = Z.prove_gkr_matmul(inp, w, n_queries=10)
    assert [hex(x) for x in proof.calldata] == g["calldata_hex"]
    assert proof.io_commitment == int(g["io_commitment"], 16)
    assert proof.final_digest == int(g["final_channel_digest"], 16)
    ok, dig = O.verify_gkr_matmul(np.array([g["input"]], np.uint32), np.array(g["weight"], np.uint32), proof.raw)
    assert ok and dig == proof.final_digest


@pytest.mark.parametrize("m,k,n", [(1, 4, 2), (2, 3, 5), (3, 16, 1), (4, 33, 20), (1, 576, 1536)],
                         ids=lambda x: str(x))
def test_gkr_matmul_matches_oracle_and_verifies(m, k, n):
    inp = int_matrix_m31(m, k, 51)
    w = int_matrix_m31(k, n, 52)
    ref = O.prove_gkr_matmul(inp, w, cap=1 << 20)
    got = Z.prove_gkr_matmul(Z.M31Matrix.from_numpy(inp), Z.M31Matrix.from_numpy(w))
    assert got.calldata == ref["calldata"]
    assert got.final_digest == ref["digest"] and got.io_commitment == ref["io"]
    ok, _ = O.verify_gkr_matmul(inp, w, got.raw)
    assert ok


def test_gkr_matmul_with_policy_commitment():
    inp = int_matrix_m31(2, 8, 61)
    w = int_matrix_m31(8, 4, 62)
    pol = Z.poseidon_hash_many([0x504F4C01] + [0] * 14)
    ref = O.prove_gkr_matmul(inp, w, policy=pol)
    got = Z.prove_gkr_matmul(Z.M31Matrix.from_numpy(inp), Z.M31Matrix.from_numpy(w), policy_commitment=pol)
    assert got.calldata == ref["calldata"] and got.final_digest == ref["digest"]
    ok, _ = O.verify_gkr_matmul(inp, w, got.raw, policy=pol)
    assert ok
