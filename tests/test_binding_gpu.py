"""GPU parity for the aggregated weight binding: the weight commitment and the
serialized binding proof (mismatch sumcheck, oracle value, super-root, opening) are
bit-identical to the oracle's restatement of the reference, the final transcripts
agree, and the oracle verifier accepts the GPU proof."""
import numpy as np
import pytest

import oracle_lib as O
import zkml_b200 as Z
from helpers import int_matrix_m31, random_qm31, uniform_m31

pytestmark = pytest.mark.gpu


def honest_specs(shapes, seed, index_base=0, full_range=False):
    rng = np.random.default_rng(seed)
    specs = []
    for i, (r, c) in enumerate(shapes):
        w = uniform_m31(r * c, seed * 10 + i).reshape(r, c) if full_range else \
            int_matrix_m31(r, c, seed * 10 + i, bound=1000)
        mle = O.mle_col_major(w)
        nv = mle.shape[0].bit_length() - 1
        pt = random_qm31(nv, rng)
        specs.append((w, index_base + i, pt, O.evaluate_mle(mle, pt), O.weight_commitment(w)))
    return specs


def to_claims(specs, device=False):
    import torch
    out = []
    for w, idx, pt, val, com in specs:
        wt = torch.from_numpy(w.view(np.int32)).cuda() if device else w
        out.append(Z.AggregatedWeightClaim(wt, idx, pt, val, O.felt_int(com)))
    return out


CASES = [([(4, 8), (8, 4)], 0, False), ([(4, 8), (2, 2), (8, 16)], 0, False), ([(16, 8)], 0, False),
         ([(3, 5), (4, 4), (2, 7), (5, 3)], 4, True), ([(2, 4), (4, 2), (1, 8)], 8, False),
         ([(64, 128), (128, 64), (32, 32), (100, 60)], 0, True), ([(300, 200), (17, 33)], 2, False)]


@pytest.mark.parametrize("shapes,base,full", CASES, ids=lambda x: str(x))
def test_binding_matches_oracle(shapes, base, full):
    specs = honest_specs(shapes, len(shapes) + base, base, full)
    for w, _, _, _, com in specs:
        assert Z.weight_commitment(w) == O.felt_int(com)
    och = O.new_channel()
    O.lib().orc_ch_mix_u64(O.C.byref(och), 11)
    rc, raw = O.prove_aggregated_binding(specs, och, n_queries=5)
    assert rc == 0
    zch = Z.PoseidonChannel()
    zch.mix_u64(11)
    proof = Z.prove_aggregated_binding(to_claims(specs, device=full), zch, n_queries=5)
    assert proof.raw.size == raw.size and (proof.raw == raw).all()
    assert zch.digest() == och.digest_int()
    vch = O.new_channel()
    O.lib().orc_ch_mix_u64(O.C.byref(vch), 11)
    assert O.verify_aggregated_binding(specs, proof.raw, vch, n_queries=5)


def test_binding_rejects_wrong_commitment():
    specs = honest_specs([(4, 8), (8, 4)], 3)
    claims = to_claims(specs)
    claims[1].commitment ^= 1
    with pytest.raises(Z.InvalidArgument):
        Z.prove_aggregated_binding(claims, Z.PoseidonChannel(), n_queries=3)
