"""The reference's transformer recipe through the GPU chain driver (Activation layers included):
bit-exact against the oracle chain, both SiLU reductions (piecewise, the reference default, and
LogUp under STWO_PIECEWISE_ACTIVATION=0).  The SmolLM2-135M shape (d = 576, 9 x 64 query width,
d_ff = 1536) at two blocks; smaller shapes cover GELU / Sigmoid and the on-chain layout."""
import numpy as np
import pytest

import oracle_lib as O
import zkml_b200 as Z
from helpers import int_matrix_m31
from zkml_b200.circuits import hf_transformer_layers

pytestmark = pytest.mark.gpu


def recipe(m, d, q_dim, d_ff, blocks, seed, act="silu"):
    x = int_matrix_m31(m, d, seed, bound=127)
    layers = hf_transformer_layers(d, q_dim, d_ff, blocks,
                                   lambda i, r, c: int_matrix_m31(r, c, seed * 100 + i, bound=127), act)
    return x, layers


@pytest.mark.parametrize("logup", [False, True], ids=["piecewise", "logup"])
@pytest.mark.parametrize("m,d,q_dim,d_ff,blocks,act", [(1, 8, 8, 16, 1, "silu"), (2, 12, 16, 20, 2, "gelu"),
                                                       (3, 16, 16, 32, 1, "sigmoid")], ids=lambda x: str(x))
def test_small_transformer_chain_matches_oracle(m, d, q_dim, d_ff, blocks, act, logup):
    x, layers = recipe(m, d, q_dim, d_ff, blocks, m + d + blocks, act)
    rc, raw, dig, io = O.prove_gkr_chain(x, layers, n_queries=4, activation_logup=logup, cap=1 << 22)
    assert rc == 0
    proof = Z.prove_gkr_chain(x, layers, n_queries=4, activation_logup=logup)
    assert proof.raw.size == raw.size and (proof.raw == raw).all()
    assert proof.final_digest == dig and proof.io_commitment == io
    ok, vdig = O.verify_gkr_chain(x, layers, proof.raw, n_queries=4, activation_logup=logup)
    assert ok and vdig == proof.final_digest


@pytest.mark.parametrize("mode", ["piecewise", "logup"])
def test_smollm2_two_blocks_matches_oracle_fixture(mode):
    """Two SmolLM2-135M blocks (d 576, d_ff 1536, SiLU) against the oracle's proof, recorded by
    tests/golden/make_transformer_fixture.py (the oracle needs minutes for it)."""
    import hashlib
    import json
    from pathlib import Path
    sys_path = Path(__file__).parent / "golden"
    fx = json.loads((sys_path / "smollm2_two_blocks.json").read_text())
    x, layers = recipe(1, 576, 576, 1536, fx["blocks"], fx["seed"], "silu")
    proof = Z.prove_gkr_chain(x, layers, n_queries=fx["n_queries"], activation_logup=(mode == "logup"))
    want = fx[mode]
    assert proof.raw.size // 4 == want["felts"]
    assert hashlib.sha256(proof.raw.astype("<u8").tobytes()).hexdigest() == want["sha256"]
    assert proof.final_digest == int(want["final_digest"], 16)
    assert proof.io_commitment == int(want["io_commitment"], 16)
    if mode == "piecewise":  # the oracle's verifier replays the whole GPU proof (the default reduction)
        ok, vdig = O.verify_gkr_chain(x, layers, proof.raw, n_queries=fx["n_queries"], activation_logup=False)
        assert ok and vdig == proof.final_digest


def test_transformer_chain_v1_calldata_matches_oracle():
    x, layers = recipe(2, 8, 8, 16, 1, 7, "silu")
    for logup in (False, True):
        rc, raw, dig, io = O.prove_gkr_chain(x, layers, n_queries=4, v1_layout=True, activation_logup=logup,
                                             cap=1 << 22)
        assert rc == 0
        proof = Z.build_verify_model_gkr_calldata(0x135, x, layers, n_queries=4, activation_logup=logup)
        got = proof.raw
        # the GPU calldata starts with model id, raw io, depth, layer count, dims and bits
        assert (got[-raw.size:] == raw).all()


def test_activation_forward_matches_oracle_on_full_range():
    """The forward pass's activation values (full M31 inputs) equal the oracle's."""
    from helpers import uniform_m31
    v = uniform_m31(4096, 99).reshape(1, 4096)
    v[0, :8] = [0, 1, 65535, 65536, (1 << 30) - 1, 1 << 30, (1 << 31) - 2, (1 << 31) - 3]
    w = np.eye(4096, dtype=np.uint32)[:, :4]
    for act in ("silu", "gelu", "sigmoid", "softmax"):
        layers = [("activation", act), ("linear", w)]
        rc, raw, dig, io = O.prove_gkr_chain(v, layers, n_queries=2, activation_logup=True, cap=1 << 22)
        assert rc == 0
        proof = Z.prove_gkr_chain(v, layers, n_queries=2, activation_logup=True)
        assert proof.io_commitment == io and proof.final_digest == dig


def test_qwen_decoder_layer_reduced_width_matches_oracle_and_verifies():
    """The config-4 layer (Qwen2.5-14B recipe: 64 tokens, 16-bit activations, SwiGLU ratio
    13824 / 5120) at a reduced width: bit-exact against the oracle with the LogUp SiLU (the
    STWO_PIECEWISE_ACTIVATION=0 pin) and accepted by the oracle's chain verifier."""
    m, d, d_ff = 64, 128, 346
    x = int_matrix_m31(m, d, 414, bound=32767)
    layers = hf_transformer_layers(d, d, d_ff, 1, lambda i, r, c: int_matrix_m31(r, c, 41400 + i, bound=127), "silu")
    rc, raw, dig, io = O.prove_gkr_chain(x, layers, n_queries=10, activation_logup=True, cap=1 << 22)
    assert rc == 0
    proof = Z.prove_gkr_chain(x, layers, n_queries=10, activation_logup=True)
    assert proof.raw.size == raw.size and (proof.raw == raw).all()
    assert proof.final_digest == dig and proof.io_commitment == io
    ok, vdig = O.verify_gkr_chain(x, layers, proof.raw, n_queries=10, activation_logup=True)
    assert ok and vdig == dig
