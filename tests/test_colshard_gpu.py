"""One matmul layer split by column blocks of the weight: the partial f_b words of the
blocks, added, give the same reduction (round polynomials, finals, next claim,
transcript) as the unsplit layer.  Ranks are emulated on one GPU here; the NCCL
version runs in test_colshard_nccl.py."""
import numpy as np
import pytest
import torch

import zkml_b200 as Z
from helpers import int_matrix_m31, log2, next_pow2, random_qm31
from zkml_b200.distributed import (column_block, reduce_matmul_layer_from_words, restrict_cols_block_words)

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("m,k,n,world", [(3, 100, 200, 2), (64, 300, 1000, 4), (8, 5120, 13824, 8), (1, 64, 128, 2),
                                         (16, 257, 700, 8)])
def test_column_blocks_equal_whole_layer(m, k, n, world):
    a = int_matrix_m31(m, k, 31)
    b = int_matrix_m31(k, n, 32)
    rng = np.random.default_rng(m + k + n)
    nv = log2(next_pow2(m)) + log2(next_pow2(n))
    point, value = random_qm31(nv, rng), random_qm31(1, rng)[0]
    ref_ch = Z.PoseidonChannel()
    ref, ref_claim = Z.reduce_matmul_layer_with_backend(Z.GKRClaim(point, value), Z.M31Matrix.from_numpy(a),
                                                        Z.M31Matrix.from_numpy(b), m, k, n, ref_ch)
    total = None
    for g in range(world):
        lo, hi = column_block(n, g, world)
        blk = torch.from_numpy(np.ascontiguousarray(b[:, lo:hi]).view(np.int32)).cuda() if hi > lo else None
        w = restrict_cols_block_words(blk, k, lo, point[log2(next_pow2(m)):])
        total = w if total is None else total + w
    ch = Z.PoseidonChannel()
    red, claim = reduce_matmul_layer_from_words(Z.GKRClaim(point, value), Z.M31Matrix.from_numpy(a), total, m, k, n,
                                                ch)
    assert ch.digest() == ref_ch.digest()
    assert (red.final_a_eval == ref.final_a_eval).all() and (red.final_b_eval == ref.final_b_eval).all()
    assert (claim.point == ref_claim.point).all() and (claim.value == ref_claim.value).all()
    for p, q in zip(red.round_polys, ref.round_polys):
        assert (p.c0 == q.c0).all() and (p.c1 == q.c1).all() and (p.c2 == q.c2).all()


def test_column_block_rejects_misaligned_offset():
    b = torch.zeros((8, 32), dtype=torch.int32, device="cuda")
    with pytest.raises(Z.InvalidArgument):
        restrict_cols_block_words(b, 8, 32, random_qm31(7, np.random.default_rng(0)))
