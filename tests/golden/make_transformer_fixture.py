"""Oracle fixture for the two-block SmolLM2-135M-shaped transformer chain.

The oracle (the C restatement of the reference prover, test infrastructure) takes minutes for
this proof, too long to rerun in every GPU test; this script runs it once and records a SHA-256
of the serialized proof (serialize_gkr_model_proof, 4 x u64 limbs per felt, little endian), its
felt count, the final channel digest and the io commitment, for both SiLU reductions.  The
inputs come from tests/helpers.py's seeded generator: input 1 x 576 and the weights int8 in
M31, the recipe of zkml_b200.circuits.hf_transformer_layers with two blocks.

Usage: python tests/golden/make_transformer_fixture.py
"""
import hashlib
import json
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
sys.path[:0] = [str(HERE.parent), str(HERE.parents[1] / "stwo-ml_b200")]

import oracle_lib as O  # noqa: E402
from helpers import int_matrix_m31  # noqa: E402
from zkml_b200.circuits import hf_transformer_layers  # noqa: E402

SEED, BLOCKS, N_QUERIES = 135, 2, 10


def case():
    x = int_matrix_m31(1, 576, SEED, bound=127)
    layers = hf_transformer_layers(576, 576, 1536, BLOCKS,
                                   lambda i, r, c: int_matrix_m31(r, c, SEED * 100 + i, bound=127), "silu")
    return x, layers


def main():
    x, layers = case()
    out = {"seed": SEED, "blocks": BLOCKS, "n_queries": N_QUERIES}
    for mode, logup in (("piecewise", False), ("logup", True)):
        rc, raw, dig, io = O.prove_gkr_chain(x, layers, n_queries=N_QUERIES, activation_logup=logup, cap=1 << 22)
        assert rc == 0, rc
        out[mode] = {"sha256": hashlib.sha256(raw.astype("<u8").tobytes()).hexdigest(), "felts": int(raw.size // 4),
                     "final_digest": hex(dig), "io_commitment": hex(io)}
        print(mode, out[mode], flush=True)
    (HERE / "smollm2_two_blocks.json").write_text(json.dumps(out, indent=1) + "\n")


if __name__ == "__main__":
    main()
