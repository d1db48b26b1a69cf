"""GPU parity for DAG circuits (Add / Mul layers, deferred skip-branch MatMul proofs) and the
verify_model_gkr calldata builder: bit-exact against the oracle in both output layouts, and
the GPU-built calldata reproduces the reference's d9_verify_gkr_calldata.txt artifact."""
import json
from pathlib import Path

import numpy as np
import pytest

import oracle_lib as O
import zkml_b200 as Z
from helpers import int_matrix_m31
from test_oracle_dag import d11_model, drop_piecewise_flag, felts, mul_circuit, sp3_model

pytestmark = pytest.mark.gpu
GOLD = json.loads((Path(__file__).parent / "golden" / "reference_vectors.json").read_text())


def test_gpu_verify_calldata_reproduces_d9():
    g = GOLD["d9_verify_calldata"]
    x, layers, y = sp3_model()
    proof = Z.build_verify_model_gkr_calldata(int(g["model_id"], 16), x, layers, n_queries=g["n_queries"])
    cd = proof.calldata
    head = 2 + cd[1] + 2 + 1 + cd[2 + cd[1] + 2] + 1  # model_id, raw io, depth, layers, dims, dequantize bits
    assert cd[:head] + drop_piecewise_flag(cd[head:]) == [int(h, 16) for h in g["calldata"]]


def residual_gated_block(seed, m=4, d=64, f=128):
    """Linear -> ReLU -> Linear -> add_from(layer 0) -> gate Linear, up Linear (from the Add)
    -> mul_from(gate) -> down Linear: the walk defers the gate branch and the residual."""
    x = int_matrix_m31(m, d, seed, bound=40)
    w = lambda r, c, i: int_matrix_m31(r, c, seed * 10 + i, bound=7)  # noqa: E731
    return x, [("linear", w(d, d, 0)), ("relu", None), ("linear", w(d, d, 2)), ("add", 0),
               ("linear", w(d, f, 4)), ("linear", w(d, f, 5), 3), ("mul", 4), ("linear", w(f, d, 7))]


def norms_block(seed, m=4, d=32):
    """Linear -> RMSNorm -> Linear -> LayerNorm -> add_from(layer 0)."""
    x = int_matrix_m31(m, d, seed, bound=60)
    w = lambda i: int_matrix_m31(d, d, seed * 10 + i, bound=5)  # noqa: E731
    return x, [("linear", w(0)), ("rmsnorm", None), ("linear", w(2)), ("layernorm", None), ("add", 0)]


CASES = {
    "d11": lambda: d11_model(),
    "mul": lambda: mul_circuit(3),
    "mul_wide": lambda: mul_circuit(11, m=8, d=32, e=16),
    "residual_gated": lambda: residual_gated_block(5),
    "residual_gated_ragged": lambda: residual_gated_block(6, m=3, d=40, f=72),
    "norms": lambda: norms_block(7),
}


@pytest.mark.parametrize("case", list(CASES))
@pytest.mark.parametrize("v1", [False, True], ids=["model_proof", "v1"])
def test_gpu_dag_matches_oracle(case, v1):
    x, layers = CASES[case]()
    rc, raw, dig, io = O.prove_gkr_chain(x, layers, n_queries=6, v1_layout=v1)
    assert rc == 0
    proof = Z.prove_gkr_chain(x, layers, n_queries=6, v1_layout=v1)
    assert proof.raw.size == raw.size and (proof.raw == raw).all()
    assert proof.final_digest == dig and proof.io_commitment == io


def test_gpu_dag_rmsnorm_residual():
    x = int_matrix_m31(4, 32, 9, bound=60)
    layers = [("linear", int_matrix_m31(32, 32, 90, bound=5)), ("rmsnorm", None),
              ("linear", int_matrix_m31(32, 32, 91, bound=5)), ("add", 0)]
    rc, raw, dig, io = O.prove_gkr_chain(x, layers, n_queries=6)
    assert rc == 0
    proof = Z.prove_gkr_chain(x, layers, n_queries=6)
    assert (proof.raw == raw).all() and proof.final_digest == dig


def test_gpu_deferred_non_linear_rejected():
    x = int_matrix_m31(2, 8, 5, bound=30)
    layers = [("linear", int_matrix_m31(8, 8, 6, bound=9)), ("relu", None),
              ("linear", int_matrix_m31(8, 8, 7, bound=9)), ("mul", 1)]
    with pytest.raises(Z.InvalidArgument):
        Z.prove_gkr_chain(x, layers, n_queries=4)


def test_gpu_verify_calldata_reproduces_d7():
    g = GOLD["d7_verify_calldata"]
    x = np.array([[1, 2, 3, 4]], np.uint32)
    w = np.array([[2 * i + j + 1 for j in range(2)] for i in range(4)], np.uint32)
    proof = Z.build_verify_model_gkr_calldata(int(g["model_id"], 16), x, [("linear", w)], n_queries=10)
    assert proof.calldata == [int(h, 16) for h in g["calldata"]]


@pytest.mark.parametrize("name", ["d9", "d11"])
def test_gpu_register_calldata_reproduced(name):
    """register_model_gkr calldata from the GPU proof's own weight commitments."""
    ref = GOLD["register_calldata"][name]
    x, layers = (sp3_model()[:2] if name == "d9" else d11_model())
    proof = Z.build_verify_model_gkr_calldata(int(ref[0], 16), x, layers, n_queries=5)
    coms = Z.verify_calldata_weight_commitments(proof.calldata, layers)
    assert Z.build_register_gkr_calldata(int(ref[0], 16), coms, layers) == ref
