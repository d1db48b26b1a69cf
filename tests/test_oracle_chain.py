"""The oracle's GKR walk over Linear / ReLU chains, pinned to the reference's own
artifacts: engine/tests/artifacts/sp3_mlp_proof.json (Linear -> ReLU -> Linear, 780
felts: every round polynomial, the ReLU bit-decomposition proof, both weight
commitments and openings with their Fiat-Shamir query indices, the io commitment)
and sp3_matmul_only_proof.json (one Linear layer)."""
import json
from pathlib import Path

import numpy as np

import oracle_lib as O

GOLD = json.loads((Path(__file__).parent / "golden" / "reference_vectors.json").read_text())


def felts(raw):
    return [O.felt_int(raw[4 * i:4 * i + 4]) for i in range(raw.size // 4)]


def test_chain_reproduces_sp3_mlp_artifact():
    g = GOLD["sp3_mlp"]
    x = np.array([g["input"]], np.uint32)
    w0, w2 = (np.array(w, np.uint32) for w in g["weights"])
    # The artifact predates the multiplicity-sumcheck / piecewise flags of the Activation
    # record and was made with 5 MLE-opening queries.
    rc, raw, dig, io = O.prove_gkr_chain(x, [("linear", w0), ("relu", None), ("linear", w2)], n_queries=5,
                                         legacy_layout=True)
    assert rc == 0
    assert felts(raw) == [int(h, 16) for h in g["calldata_hex"]]
    assert io == int(g["io_commitment"], 16)
    assert felts(raw)[-1] == io


def test_chain_current_layout_adds_the_two_record_flags():
    g = GOLD["sp3_mlp"]
    x = np.array([g["input"]], np.uint32)
    w0, w2 = (np.array(w, np.uint32) for w in g["weights"])
    rc, raw, _, _ = O.prove_gkr_chain(x, [("linear", w0), ("relu", None), ("linear", w2)], n_queries=5)
    rc2, raw2, _, _ = O.prove_gkr_chain(x, [("linear", w0), ("relu", None), ("linear", w2)], n_queries=5,
                                        legacy_layout=True)
    f, f2 = felts(raw), felts(raw2)
    assert rc == rc2 == 0 and len(f) == len(f2) + 2
    assert f[39] == 0 and f[:39] == f2[:39]


def test_chain_reproduces_sp3_matmul_only_artifact():
    g = GOLD["sp3_matmul_only"]
    x = np.array([g["input"]], np.uint32)
    w = np.array(g["weight"], np.uint32)
    rc, raw, dig, io = O.prove_gkr_chain(x, [("linear", w)])
    assert rc == 0
    assert felts(raw) == [int(h, 16) for h in g["calldata_hex"]]
    assert dig == int(g["final_channel_digest"], 16) and io == int(g["io_commitment"], 16)
