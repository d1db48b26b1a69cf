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


def test_chain_with_rmsnorm_runs_and_is_deterministic():
    rng_w = [np.arange(64, dtype=np.uint32).reshape(8, 8) % 13, np.arange(32, dtype=np.uint32).reshape(8, 4) % 7]
    x = (np.arange(16, dtype=np.uint32).reshape(2, 8) * 37) % 200
    layers = [("rmsnorm", None), ("linear", rng_w[0]), ("relu", None), ("linear", rng_w[1]), ("rmsnorm", None)]
    rc, raw, dig, io = O.prove_gkr_chain(x, layers, n_queries=3)
    rc2, raw2, dig2, io2 = O.prove_gkr_chain(x, layers, n_queries=3)
    assert rc == rc2 == 0 and (raw == raw2).all() and dig == dig2
    f = [O.felt_int(raw[4 * i:4 * i + 4]) for i in range(raw.size // 4)]
    assert f[0] == len(layers) and f[1] == 8  # first record is the output RMSNorm (tag 8)


def test_oracle_transformer_chain_verifies_and_rejects_tampering():
    """The oracle's chain verifier (verify_gkr's walk, restated) accepts the oracle's transformer
    proofs with both SiLU reductions and ends on the prover's digest; a flipped felt is rejected."""
    import sys
    from pathlib import Path
    sys.path.insert(0, str(Path(__file__).resolve().parents[1] / "stwo-ml_b200"))
    from helpers import int_matrix_m31
    from zkml_b200.circuits import hf_transformer_layers
    x = int_matrix_m31(2, 8, 1)
    for act, logup in (("silu", False), ("silu", True), ("gelu", False), ("sigmoid", True)):
        layers = hf_transformer_layers(8, 8, 16, 2, lambda i, r, c: int_matrix_m31(r, c, 100 + i), act)
        rc, raw, dig, io = O.prove_gkr_chain(x, layers, n_queries=4, activation_logup=logup, cap=1 << 22)
        assert rc == 0
        ok, vdig = O.verify_gkr_chain(x, layers, raw, n_queries=4, activation_logup=logup)
        assert ok and vdig == dig
        for pos in (4 * 3, 4 * 150, raw.size - 8):
            bad = raw.copy()
            bad[pos] ^= 1
            assert not O.verify_gkr_chain(x, layers, bad, n_queries=4, activation_logup=logup)[0]
