"""GPU parity for the algebraic ReLU reduction and the GKR chain driver: bit-exact
against the oracle, and the whole GPU chain proof reproduces the reference's
sp3_mlp_proof.json artifact (Linear -> ReLU -> Linear, 780 felts)."""
import json
from pathlib import Path

import numpy as np
import pytest

import oracle_lib as O
import zkml_b200 as Z
from helpers import int_matrix_m31, random_qm31, uniform_m31

pytestmark = pytest.mark.gpu
GOLD = json.loads((Path(__file__).parent / "golden" / "reference_vectors.json").read_text())


@pytest.mark.parametrize("rows,cols", [(1, 2), (1, 4), (2, 3), (4, 16), (3, 5), (16, 100), (64, 1024)],
                         ids=lambda x: str(x))
def test_relu_matches_oracle(rows, cols):
    x = uniform_m31(rows * cols, rows * 5 + cols).reshape(rows, cols)
    rng = np.random.default_rng(rows + cols)
    nv = (rows - 1).bit_length() + (cols - 1).bit_length()
    point, value = random_qm31(nv, rng), random_qm31(1, rng)[0]
    och = O.new_channel()
    rc, raw, ie, nxt = O.reduce_activation_relu(x, point, value, och)
    assert rc == 0
    zch = Z.PoseidonChannel()
    proof, claim = Z.reduce_activation_layer_relu(Z.GKRClaim(point, value), Z.M31Matrix.from_numpy(x), zch)
    assert proof.raw.size == raw.size and (proof.raw == raw).all()
    assert (claim.value == ie).all() and (claim.point == nxt).all()
    assert zch.digest() == och.digest_int()


def test_gpu_chain_reproduces_sp3_mlp_artifact():
    g = GOLD["sp3_mlp"]
    x = np.array([g["input"]], np.uint32)
    w0, w2 = (np.array(w, np.uint32) for w in g["weights"])
    proof = Z.prove_gkr_chain(x, [("linear", w0), ("relu", None), ("linear", w2)], n_queries=5,
                              legacy_activation_record=True)
    assert proof.calldata == [int(h, 16) for h in g["calldata_hex"]]
    assert proof.io_commitment == int(g["io_commitment"], 16)


def chain_case(m, dims, seed):
    rng = np.random.default_rng(seed)
    x = int_matrix_m31(m, dims[0], seed, bound=50)
    layers = []
    for i in range(1, len(dims)):
        layers.append(("linear", int_matrix_m31(dims[i - 1], dims[i], seed * 10 + i, bound=20)))
        if i + 1 < len(dims):
            layers.append(("relu", None))
    return x, layers


@pytest.mark.parametrize("m,dims", [(1, [4, 4, 2]), (2, [8, 16, 4]), (3, [5, 7, 6, 3]), (8, [64, 128, 64]),
                                    (1, [576, 1536, 576])], ids=lambda x: str(x))
def test_gpu_chain_matches_oracle(m, dims):
    x, layers = chain_case(m, dims, m + len(dims))
    rc, raw, dig, io = O.prove_gkr_chain(x, layers, n_queries=6)
    assert rc == 0
    proof = Z.prove_gkr_chain(x, layers, n_queries=6)
    assert proof.raw.size == raw.size and (proof.raw == raw).all()
    assert proof.final_digest == dig and proof.io_commitment == io


def norm_chain_case(m, d, d_ff, seed):
    """One SmolLM-style block of the reference recipe (hf_loader.rs:770-813) with the gated FFN
    replaced by Linear -> ReLU -> Linear: RMSNorm, q, o, RMSNorm, up, ReLU, down, final RMSNorm."""
    x = int_matrix_m31(m, d, seed, bound=100)
    w = [int_matrix_m31(a, b, seed * 10 + i, bound=20) for i, (a, b) in enumerate([(d, d), (d, d), (d, d_ff),
                                                                                     (d_ff, d)])]
    layers = [("rmsnorm", None), ("linear", w[0]), ("linear", w[1]), ("rmsnorm", None), ("linear", w[2]),
              ("relu", None), ("linear", w[3]), ("rmsnorm", None)]
    return x, layers


@pytest.mark.parametrize("m,d,d_ff", [(2, 8, 16), (3, 12, 20), (1, 576, 1536)], ids=lambda x: str(x))
def test_gpu_chain_with_rmsnorm_matches_oracle(m, d, d_ff):
    x, layers = norm_chain_case(m, d, d_ff, m + d)
    rc, raw, dig, io = O.prove_gkr_chain(x, layers, n_queries=4)
    assert rc == 0
    proof = Z.prove_gkr_chain(x, layers, n_queries=4)
    assert proof.raw.size == raw.size and (proof.raw == raw).all()
    assert proof.final_digest == dig and proof.io_commitment == io
