"""The sumcheck round schedules give the same proofs.

The restriction has a tensor-pipe and a generic kernel, the row side a fused
launch (up to 2^8 rows; the last two shapes sit on either side of that bound), a
second-stream and a same-stream form, and the round loop has four schedules
(look-ahead rounds queued up front with a resident-block tail; queued without the
tail; launched one at a time; and the plain fold-and-sum rounds), the queued ones
with or without programmatic dependent launches.  Each is selected by environment variables read
when a context is created, so every schedule runs in its own process and is
checked against the oracle on products that stay small, cross the look-ahead
threshold, and matrices that go through the restrictions.
"""
import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]

SCRIPT = r"""
import sys
import numpy as np
sys.path[:0] = [{root!r}, {root!r} + "/tests", {root!r} + "/stwo-ml_b200"]
import zkml_b200 as Z
import oracle_lib
from helpers import int_matrix_m31, uniform_m31
be = Z.GpuBackend(0)
rng = np.random.default_rng(4)
def check(a, b, r_i, r_j):
    m, k = a.shape
    n = b.shape[1]
    pk = 1 << max(0, (k - 1).bit_length())
    got = be.reduce_matmul_layer(Z.M31Matrix.from_numpy(a), Z.M31Matrix.from_numpy(b), r_i, r_j, pk, Z.PoseidonChannel())
    ref = oracle_lib.reduce_matmul_layer(a, b, r_i, r_j, oracle_lib.new_channel(), mode=0, nthreads=4)
    rp = np.stack([np.concatenate([p.c0, p.c1, p.c2]) for p in got.round_polys]) if got.round_polys else np.zeros((0, 12), np.uint32)
    assert (rp == ref["round_polys"]).all(), (m, k, n)
    assert (got.challenges == ref["challenges"]).all()
    assert (got.final_a_eval == ref["final_a"]).all() and (got.final_b_eval == ref["final_b"]).all()
for lg in (1, 2, 5, 11, 12, 17):
    n = 1 << lg
    check(uniform_m31(n, lg).reshape(1, n), uniform_m31(n, lg + 50).reshape(n, 1), np.zeros((0, 4), np.uint32), np.zeros((0, 4), np.uint32))
for (m, k, n) in ((4, 96, 80), (8, 3000, 64), (2, 8192, 16), (3, 37, 1028), (16, 300, 2052), (5, 17, 6),
                  (2, 33, 4100), (4, 1000, 3072), (256, 64, 96), (300, 40, 70)):
    a = int_matrix_m31(m, k, 1)
    b = int_matrix_m31(k, n, 2)
    lm = (m - 1).bit_length()
    ln = (n - 1).bit_length()
    check(a, b, rng.integers(0, 2**31 - 1, (lm, 4), dtype=np.uint32), rng.integers(0, 2**31 - 1, (ln, 4), dtype=np.uint32))
print("ok")
"""

MODES = {
    "queued_tail": {},
    "queued_no_tail": {"ZKML_LOOKAHEAD_TAIL": "0"},
    "unqueued": {"ZKML_LA_QUEUE": "0"},
    "plain_rounds": {"ZKML_LOOKAHEAD_MAX": "0"},
    "generic_restriction": {"ZKML_RESTRICT_TC": "0"},
    "plain_dependent_launches": {"ZKML_LA_PDL": "0"},
    "rows_unfused_side_stream": {"ZKML_ROWS_FUSED": "0"},
    "rows_unfused_one_stream": {"ZKML_ROWS_FUSED": "0", "ZKML_ROW_SIDE_STREAM": "0"},
}


@pytest.mark.gpu
@pytest.mark.parametrize("mode", sorted(MODES))
def test_round_schedules_match_oracle(mode):
    env = dict(os.environ)
    env.update(MODES[mode])
    r = subprocess.run([sys.executable, "-c", SCRIPT.format(root=str(ROOT))], env=env, capture_output=True,
                       text=True, timeout=600)
    assert r.returncode == 0 and r.stdout.strip().endswith("ok"), r.stdout[-2000:] + r.stderr[-4000:]


@pytest.mark.gpu
def test_queued_round_kernel_wait_is_bounded():
    """A queued round kernel whose challenge never comes gives up and flags it."""
    sys.path[:0] = [str(ROOT / "stwo-ml_b200")]
    import zkml_b200 as Z
    ctx = Z.Context(0)
    st = np.zeros(1, np.uint32)
    Z._check(Z.lib().zkml_selftest_wait_timeout(ctx.handle, st))
    assert st[0] == 1
    # the context keeps working afterwards
    from zkml_b200.distributed import GpuSumcheckSession
    sess = GpuSumcheckSession(ctx)
    sess.load_m31(np.arange(1, 17, dtype=np.uint32), np.arange(1, 17, dtype=np.uint32))
    w = sess.round(None)
    assert w.shape == (12,)
    ctx.close()
