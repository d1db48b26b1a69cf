"""The allocation-free column restriction (zkml_restrict_cols_noalloc).

It exists for callers that cannot allocate GPU memory; its scratch is a fixed
array inside the library.  Checked through the C ABI against the existing
ZkmlOps::restrict_mle entry point and against the CPU oracle's restrict_mle
(backend.rs:199-215), both applied to the column-major padded MLE of the same
matrix -- the same f_b, bit for bit -- on two calls in a row (the shared array
keeps the first call's contents, which the second must not see).  The shapes
cover a column count below 64 (no high eq variables) and one above 65536 (the
high eq table no longer fits the kernel's shared-memory copy).
Collected last so that a run stopping at the first failure has run everything
else first.
"""
import numpy as np
import pytest

import oracle_lib as O
import zkml_b200 as Z
from helpers import int_matrix_m31, log2, next_pow2, random_qm31, uniform_m31

pytestmark = pytest.mark.gpu


def colmajor_padded_mle(b):
    rows, cols = b.shape
    pr, pc = next_pow2(rows), next_pow2(cols)
    mle = np.zeros((pc, pr, 4), np.uint32)
    mle[:cols, :rows, 0] = b.T
    return mle.reshape(-1, 4)


def reference_restriction(b, r_j):
    # existing entry point: ZkmlOps::restrict_mle on the column-major MLE
    return Z.GpuBackend(0).restrict_mle(colmajor_padded_mle(b), r_j)


def oracle_restriction(b, r_j):
    return O.restrict_mle(colmajor_padded_mle(b), r_j)


def run_noalloc(b, r_j):
    import torch
    rows, cols = b.shape
    tb = torch.from_numpy(b.view(np.int32)).cuda()
    out = torch.full((next_pow2(rows), 4), -1, dtype=torch.int32, device="cuda")
    Z.restrict_cols_noalloc(tb, rows, cols, r_j, out)
    torch.cuda.synchronize()
    return out.cpu().numpy().view(np.uint32)


def test_noalloc_restriction_matches_existing_entry_twice():
    rng = np.random.default_rng(11)
    b1 = int_matrix_m31(300, 200, 71)
    r1 = random_qm31(log2(next_pow2(200)), rng)
    b2 = uniform_m31(257 * 1000, 72).reshape(257, 1000)
    r2 = random_qm31(log2(next_pow2(1000)), rng)
    got1 = run_noalloc(b1, r1)
    got2 = run_noalloc(b2, r2)
    for b, r, got in ((b1, r1, got1), (b2, r2, got2)):
        want = oracle_restriction(b, r)
        assert (got == want).all()
        assert (got == reference_restriction(b, r)).all()


@pytest.mark.parametrize("rows,cols,seed", [(5, 37, 81), (4, 70000, 82), (3, 1, 83)])
def test_noalloc_narrow_and_wide_columns(rows, cols, seed):
    rng = np.random.default_rng(seed)
    b = uniform_m31(rows * cols, seed).reshape(rows, cols)
    r = random_qm31(log2(next_pow2(cols)), rng)
    for _ in range(2):
        assert (run_noalloc(b, r) == oracle_restriction(b, r)).all()


def test_noalloc_rejects_oversize_and_bad_values():
    import torch
    small = torch.zeros((4, 4), dtype=torch.int32, device="cuda")
    out = torch.zeros((8, 4), dtype=torch.int32, device="cuda")
    with pytest.raises(Z.InvalidArgument):
        Z.restrict_cols_noalloc(small, Z.NOALLOC_MAX_ROWS + 1, 4, np.zeros((2, 4), np.uint32), out)
    bad = torch.from_numpy(np.full((4, 4), 0x80000001, np.uint32).view(np.int32)).cuda()
    with pytest.raises(Z.InvalidArgument):
        Z.restrict_cols_noalloc(bad, 4, 4, np.zeros((2, 4), np.uint32), out)
    # the shared array is still usable afterwards
    rng = np.random.default_rng(3)
    b = int_matrix_m31(8, 64, 5)
    r = random_qm31(6, rng)
    assert (run_noalloc(b, r) == oracle_restriction(b, r)).all()
