"""The CPU oracle against the reference's own golden vectors (no GPU)."""
import json
from pathlib import Path

import numpy as np
import pytest

import oracle_lib as O

GOLD = json.loads((Path(__file__).parent / "golden" / "reference_vectors.json").read_text())


@pytest.mark.parametrize("kat", GOLD["poseidon_kats"], ids=lambda k: k["op"])
def test_poseidon_kats(kat):
    xs = [int(x, 16) for x in kat["inputs"]]
    if kat["op"] == "poseidon_hash":
        got = O.poseidon_hash(*xs)
    else:
        got = O.poseidon_hash_many(xs)
    assert got == int(kat["expect"], 16)


def test_hades_matches_poseidon_hash():
    # engine/src/crypto/hades.rs:60-75: hades([x, y, 2])[0] == poseidon_hash(x, y)
    st = np.concatenate([O.felt(42), O.felt(99), O.felt(2)])
    O.lib().orc_hades(st)
    assert O.felt_int(st[:4]) == O.poseidon_hash(42, 99)


def test_sp3_matmul_only_artifact_bit_exact():
    g = GOLD["sp3_matmul_only"]
    inp = np.array([g["input"]], np.uint32)
    w = np.array(g["weight"], np.uint32)
    res = O.prove_gkr_matmul(inp, w, policy=None, n_queries=10)
    assert [hex(x) for x in res["calldata"]] == g["calldata_hex"]
    assert res["io"] == int(g["io_commitment"], 16)
    assert res["digest"] == int(g["final_channel_digest"], 16)
    ok, dig = O.verify_gkr_matmul(inp, w, res["raw"])
    assert ok and dig == res["digest"]


def test_sp3_weight_opening_calldata():
    g = GOLD["sp3_matmul_only"]
    res = O.prove_gkr_matmul(np.array([g["input"]], np.uint32), np.array(g["weight"], np.uint32))
    cd = [hex(x) for x in res["calldata"]]
    wo = g["weight_opening_calldata_hex"]
    # The standalone opening calldata is [count, opening...]; inside the GKR calldata the
    # opening follows the weight claim (eval point + expected value).
    assert wo[0] == "0x1"
    body = wo[1:]
    start = len(cd) - 1 - len(body)
    assert cd[start:start + len(body)] == body


def test_verifier_rejects_tamper():
    g = GOLD["sp3_matmul_only"]
    inp = np.array([g["input"]], np.uint32)
    w = np.array(g["weight"], np.uint32)
    res = O.prove_gkr_matmul(inp, w)
    raw = res["raw"].copy()
    raw[4 * 3] ^= 1  # first round c0.a
    ok, _ = O.verify_gkr_matmul(inp, w, raw)
    assert not ok
