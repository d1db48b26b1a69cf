"""Extract the golden vectors the parity tests pin against.

Reads the reference checkout (available only where it is mounted) and writes
``reference_vectors.json`` next to this script.  The vectors are the
reference's own known answers for the matmul-sumcheck path:

* ``sp3_matmul_only``: engine/tests/artifacts/sp3_matmul_only_proof.json,
  produced by engine/tests/e2e_cairo_verify.rs:1093-1180 (1x4 input [1,2,3,4],
  weight W[i][j] = 2i+j+1, 4x2) -- full GKR calldata, weight commitment,
  weight claims, weight-opening calldata, io commitment, final channel digest.
* ``sp3_mlp``: engine/tests/artifacts/sp3_mlp_proof.json, produced by
  engine/tests/e2e_cairo_verify.rs:978-1040 from build_gkr_mlp_relu (272-304): 1x4 input
  [1,2,3,4] -> Linear(4) with W0[i][j] = (i+j)%7+1 -> ReLU -> Linear(2) with
  W2[i][j] = i+j+1 -- full GKR calldata (780 felts), weight commitments, io commitment,
  final channel digest.
* ``d9_verify_calldata``: engine/tests/artifacts/d9_verify_gkr_calldata.txt, written by
  engine/tests/e2e_cairo_verify.rs:1375-1470 (build_verify_model_gkr_calldata, layout V1, for
  the sp3_mlp model with model id 0xd9) -- the whole verify_model_gkr calldata (754 felts).
  The artifact was generated with 5 MLE-opening queries (its opening proofs carry 5) and
  predates the Activation record's trailing piecewise flag (cairo_serde.rs:1881).
* ``d7_verify_calldata``: engine/tests/artifacts/d7_verify_gkr_calldata.txt, written by
  e2e_cairo_verify.rs:1294-1370 for the sp3_matmul_only model (model id 0xd7): the whole V1
  verify_model_gkr calldata (236 felts).
* ``register_calldata``: the d7 / d9 / d11 register_model_gkr calldata (build_register_gkr_calldata,
  starknet.rs:1619-1640: model id, the walk's weight commitments, the circuit descriptor).
* ``d10_weight_commitments``: d10_onchain_summary.json (Linear(identity) -> LayerNorm ->
  Linear(4->2) on [[7,9,11,13],[17,19,21,23]], e2e_cairo_verify.rs:312-352); the rest of the
  d10 artifacts predate the current rsqrt table, so only the weight commitments are pinned.
* ``d11_residual``: engine/tests/artifacts/d11_verify_gkr_calldata.txt and
  d11_onchain_summary.json, written by e2e_cairo_verify.rs:1549-1660 for
  Linear(identity 4x4) -> fork -> ReLU -> Linear(W2[i][j] = (i+j)%3+1) -> add_from(fork) on the
  input [1,2,3,4] (model id 0xdb).  The calldata file predates the compressed round
  polynomials (it carries c0, c1, c2) and the algebraic ReLU proof, so only its leading Add
  record and the first round of the next MatMul are pinned, with the io commitment and the
  walk's weight commitments.
* ``poseidon_kats``: engine/src/crypto/poseidon_channel.rs:1619-1637
  (poseidon_hash_many([0, pack(QM31(1,2,3,4))])) and
  stwo-gpu/crates/stwo/src/core/channel/poseidon252.rs:230-241
  (Poseidon252Channel::mix_u64(0x1111222233334444) from the zero digest,
  i.e. poseidon_hash(0, 0x1111222233334444)).

Usage: python tests/golden/make_golden.py <reference root>
"""
import json
import sys
from pathlib import Path

if len(sys.argv) != 2:
    sys.exit("usage: make_golden.py <reference checkout root>")
ref = Path(sys.argv[1])
art = json.loads((ref / "engine/tests/artifacts/sp3_matmul_only_proof.json").read_text())
mlp = json.loads((ref / "engine/tests/artifacts/sp3_mlp_proof.json").read_text())
d11_summary = json.loads((ref / "engine/tests/artifacts/d11_onchain_summary.json").read_text())


def _calldata(name):
    """The artifact's felts as hex strings (decimal tokens converted)."""
    toks = (ref / f"engine/tests/artifacts/{name}_verify_gkr_calldata.txt").read_text().split()
    return [t if t.startswith("0x") else hex(int(t)) for t in toks]


def _d11_proof_data():
    """proof_data of the d11 calldata: after model_id, raw io, depth, layer count, matmul
    dims (6) and dequantize bits (0) comes its length, then the felts."""
    v = [int(t, 16) for t in _calldata("d11")]
    i = 2 + v[1] + 2 + 1 + v[2 + v[1] + 2] + 1
    n = v[i]
    return [int(x) for x in v[i + 1:i + 1 + n]]

out = {
    "sp3_matmul_only": {
        "source": "engine/tests/artifacts/sp3_matmul_only_proof.json",
        "input": art["input_data"],
        "input_shape": art["model"]["input_shape"],
        "weight": [[2 * i + j + 1 for j in range(2)] for i in range(4)],
        "output": art["output_data"],
        "calldata_hex": art["calldata_hex"],
        "weight_commitments": art["weight_commitments"],
        "weight_claims": art["weight_claims"],
        "weight_opening_calldata_hex": art["weight_opening_calldata_hex"],
        "io_commitment": art["io_commitment"],
        "final_channel_digest": art["verification"]["final_channel_digest"],
    },
    "sp3_mlp": {
        "source": "engine/tests/artifacts/sp3_mlp_proof.json",
        "input": mlp["input_data"],
        "input_shape": mlp["model"]["input_shape"],
        "layers": mlp["model"]["layers"],
        "weights": [[[(i + j) % 7 + 1 for j in range(4)] for i in range(4)],
                    [[i + j + 1 for j in range(2)] for i in range(4)]],
        "output": mlp["output_data"],
        "calldata_hex": mlp["calldata_hex"],
        "weight_commitments": mlp["weight_commitments"],
        "io_commitment": mlp["io_commitment"],
        "final_channel_digest": mlp["verification"]["final_channel_digest"],
    },
    "d9_verify_calldata": {
        "source": "engine/tests/artifacts/d9_verify_gkr_calldata.txt",
        "model_id": "0xd9",
        "n_queries": 5,
        "calldata": _calldata("d9"),
    },
    "d7_verify_calldata": {
        "source": "engine/tests/artifacts/d7_verify_gkr_calldata.txt",
        "model_id": "0xd7",
        "calldata": _calldata("d7"),
    },
    "register_calldata": {
        name: (ref / f"engine/tests/artifacts/{name}_register_gkr_calldata.txt").read_text().split()
        for name in ("d7", "d9", "d11")
    },
    "d10_weight_commitments": json.loads(
        (ref / "engine/tests/artifacts/d10_onchain_summary.json").read_text())["weight_commitments"],
    "d11_residual": {
        "source": "engine/tests/artifacts/d11_verify_gkr_calldata.txt, d11_onchain_summary.json",
        "model_id": "0xdb",
        "input": [[1, 2, 3, 4]],
        "w0": [[1 if i == j else 0 for j in range(4)] for i in range(4)],
        "w2": [[(i + j) % 3 + 1 for j in range(4)] for i in range(4)],
        "add_record": _d11_proof_data()[:10],
        "matmul_round0_c0": _d11_proof_data()[12:16],
        "matmul_round0_c2": _d11_proof_data()[20:24],
        "io_commitment": d11_summary["io_commitment"],
        "weight_commitments": d11_summary["weight_commitments"],
    },
    "poseidon_kats": [
        {
            "op": "poseidon_hash_many",
            "inputs": ["0x0", "0x10000000200000008000000180000004"],
            "expect": "0x0e029e34eb10ff7719b4a23d283495d23f65760b9d9a9b7885f0350879a7f1c",
            "source": "engine/src/crypto/poseidon_channel.rs:1619-1637",
        },
        {
            "op": "poseidon_hash",
            "inputs": ["0x0", "0x1111222233334444"],
            "expect": "0x07cecc0ee3d858c843fe63165f038353f9f80f52dd8d32eead9f635e2f7d8b8e",
            "source": "stwo-gpu/crates/stwo/src/core/channel/poseidon252.rs:230-241",
        },
    ],
}
# Sanity: the KAT strings above are the ones in the reference sources.
src1 = (ref / "engine/src/crypto/poseidon_channel.rs").read_text()
src2 = (ref / "stwo-gpu/crates/stwo/src/core/channel/poseidon252.rs").read_text()
assert out["poseidon_kats"][0]["expect"] in src1
assert out["poseidon_kats"][1]["expect"] in src2
# Sanity: the MLP weights are the ones build_gkr_mlp_relu sets.
src3 = (ref / "engine/tests/e2e_cairo_verify.rs").read_text()
assert "M31::from(((i + j) % 7 + 1) as u32)" in src3 and "M31::from((i + j + 1) as u32)" in src3
# Sanity: the d11 residual model's weights are the ones its test sets.
assert "w2.set(i, j, M31::from(((i + j) % 3 + 1) as u32));" in src3 and "w0.set(i, i, M31::from(1u32));" in src3
dst = Path(__file__).with_name("reference_vectors.json")
dst.write_text(json.dumps(out, indent=1) + "\n")
print("wrote", dst)
