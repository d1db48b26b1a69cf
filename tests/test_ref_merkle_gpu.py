"""The reference's own Poseidon-252 Merkle layer kernel (oracle/_ref/libref_merkle.so, compiled
from its CUDA source by oracle/build_ref_merkle.py) against this library: the same hashes and the
same MLE commitment roots.  This pins the measuring stick that bench.py times beside the
library's Merkle kernel (skipped when the harness was not built)."""
import numpy as np
import pytest

import ref_merkle as R
import zkml_b200 as Z
from helpers import uniform_m31

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not R.available(), reason="oracle/_ref/libref_merkle.so not built")]


def _dev(torch, arr):
    return torch.from_numpy(np.ascontiguousarray(arr).view(np.int64)).cuda()


def test_reference_kernel_hashes_equal_poseidon_hash():
    import torch
    rng = np.random.default_rng(5)
    pairs = [(int(rng.integers(0, 2**62)) * 2**189 % R.STARK_P, int(rng.integers(0, 2**62))) for _ in range(64)]
    pairs[0] = (0, 0)
    pairs[1] = (R.STARK_P - 1, R.STARK_P - 2)
    children = R.limbs([v for pr in pairs for v in pr])
    rc = _dev(torch, R.limbs(R.compressed_round_keys()))
    d_in = _dev(torch, children)
    d_out = torch.zeros((64, 4), dtype=torch.int64, device="cuda")
    assert R.lib().ref_merkle_hash_level(d_in.data_ptr(), d_out.data_ptr(), 64, rc.data_ptr(), None) == 0
    torch.cuda.synchronize()
    got = d_out.cpu().numpy().view(np.uint64)
    for i, (a, b) in enumerate(pairs):
        assert sum(int(got[i, j]) << (64 * j) for j in range(4)) == Z.poseidon_hash(a, b), i


@pytest.mark.parametrize("log_n", [1, 5, 16])
def test_reference_kernel_root_equals_commit_mle_root(log_n):
    import torch
    n = 1 << log_n
    leaves = uniform_m31(4 * n, 700 + log_n).reshape(n, 4)
    rc = _dev(torch, R.limbs(R.compressed_round_keys()))
    d_leaves = _dev(torch, R.leaf_felts(leaves))
    scratch = torch.zeros((n, 4), dtype=torch.int64, device="cuda")
    assert R.lib().ref_merkle_root(d_leaves.data_ptr(), n, scratch.data_ptr(), rc.data_ptr(), None) == 0
    torch.cuda.synchronize()
    root = scratch[0].cpu().numpy().view(np.uint64)
    ours = Z.commit_mle_root(leaves)
    assert sum(int(root[j]) << (64 * j) for j in range(4)) == ours
