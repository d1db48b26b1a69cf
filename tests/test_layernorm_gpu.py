"""GPU parity for the LayerNorm reduction (reduce_layernorm_layer, gkr/prover.rs:7944-8354):
bit-exact against the oracle, standalone and inside a GKR circuit."""
import numpy as np
import pytest

import oracle_lib as O
import zkml_b200 as Z
from helpers import random_qm31, uniform_m31

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("rows,cols,dim", [(1, 2, 2), (1, 4, 4), (2, 4, 4), (3, 5, 5), (4, 16, 12), (2, 64, 64),
                                           (64, 576, 576), (8, 5120, 5120)], ids=lambda x: str(x))
def test_layernorm_matches_oracle(rows, cols, dim):
    x = uniform_m31(rows * cols, rows * 7 + cols).reshape(rows, cols) % 60000
    nv = (rows - 1).bit_length() + (cols - 1).bit_length()
    rng = np.random.default_rng(rows + cols)
    point, value = random_qm31(nv, rng), random_qm31(1, rng)[0]
    och = O.new_channel()
    rc, raw, ie = O.reduce_layernorm(x, dim, point, value, och, cap=1 << 18)
    assert rc == 0
    zch = Z.PoseidonChannel()
    proof, claim = Z.reduce_layernorm_layer(Z.GKRClaim(point, value), Z.M31Matrix.from_numpy(x), dim, zch)
    assert proof.raw.size == raw.size and (proof.raw == raw).all()
    assert (claim.value == ie).all()
    assert zch.digest() == och.digest_int()


def test_gpu_chain_with_layernorm_matches_oracle():
    x = uniform_m31(4 * 32, 9).reshape(4, 32) % 3000
    w = (uniform_m31(32 * 16, 10).reshape(32, 16) % 7).astype(np.uint32)
    layers = [("layernorm", None), ("linear", w), ("layernorm", None), ("add", 1)]
    rc, raw, dig, io = O.prove_gkr_chain(x, layers, n_queries=4)
    assert rc == 0
    proof = Z.prove_gkr_chain(x, layers, n_queries=4)
    assert (proof.raw == raw).all() and proof.final_digest == dig and proof.io_commitment == io
