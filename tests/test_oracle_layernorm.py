"""The oracle's LayerNorm reduction (reduce_layernorm_layer, gkr/prover.rs:7944-8354).

Parity unpinned: the reference's only LayerNorm artifact (d10, engine/tests/artifacts) was
written with an earlier rsqrt table (2^16 / sqrt(v) in real arithmetic; the current
build_rsqrt_table, components/layernorm.rs:116-136, uses an integer square root), so only its
weight commitments still hold; they are checked here.  The forward pass is checked against an
independent Python restatement of apply_layernorm_detailed (compiler/prove.rs:977-1060) and the
record's evaluations against MLEs of those vectors."""
import json
from pathlib import Path

import numpy as np
import pytest

import oracle_lib as O
from helpers import random_qm31, uniform_m31
from test_oracle_dag import felts

P = (1 << 31) - 1
GOLD = json.loads((Path(__file__).parent / "golden" / "reference_vectors.json").read_text())


def layernorm_ref(x, dim):
    """apply_layernorm_detailed over the padded matrix: (output, mean, var, rsqrt) per element."""
    rows, cols = x.shape
    pr, pc = 1 << (rows - 1).bit_length(), 1 << (cols - 1).bit_length()
    xp = np.zeros((pr, pc), np.int64)
    xp[:rows, :cols] = x % P
    table = O.rsqrt_table(16)
    na = min(dim, pc)
    inv = pow(na, P - 2, P)
    out, mean, var, rs = (np.zeros((pr, pc), np.int64) for _ in range(4))
    for i in range(pr):
        mu = int(sum(int(v) for v in xp[i, :na]) % P) * inv % P
        vs = sum((int(v) - mu) % P * ((int(v) - mu) % P) for v in xp[i, :na]) % P
        va = vs * inv % P & 0xFFFF
        r = int(table[va])
        for j in range(pc):
            out[i, j] = (int(xp[i, j]) - mu) % P * r % P
        mean[i], var[i], rs[i] = mu, va, r
    return out, mean, var, rs


def mle_eval(v, point):
    return O.evaluate_mle(np.stack([v.reshape(-1) % P, *[np.zeros(v.size, np.int64)] * 3], 1).astype(np.uint32),
                          point)


@pytest.mark.parametrize("rows,cols,dim", [(1, 4, 4), (2, 4, 4), (3, 5, 5), (4, 16, 12), (2, 64, 64)],
                         ids=lambda x: str(x))
def test_layernorm_record_evaluations(rows, cols, dim):
    x = uniform_m31(rows * cols, rows * 7 + cols).reshape(rows, cols) % 5000
    nv = (rows - 1).bit_length() + (cols - 1).bit_length()
    rng = np.random.default_rng(rows + cols)
    point, value = random_qm31(nv, rng), random_qm31(1, rng)[0]
    rc, raw, ie = O.reduce_layernorm(x, dim, point, value, O.new_channel())
    assert rc == 0
    f = felts(raw)
    out, mean, var, rs = layernorm_ref(x, dim)
    xp = np.zeros_like(out)
    xp[:rows, :cols] = x
    q = lambda at: f[at:at + 4]  # noqa: E731
    assert f[0] == 4
    assert q(1) == list(mle_eval(xp, point)) == list(ie)
    assert q(5) == list(mle_eval(out, point))
    assert q(9) == list(mle_eval(mean, point))
    assert q(13) == list(mle_eval(rs, point))
    assert f[18:21] == [0, 1, min(dim, 1 << (cols - 1).bit_length())]  # not SIMD, mean/var present, n_active


def test_d10_weight_commitments():
    x = np.array([[7, 9, 11, 13], [17, 19, 21, 23]], np.uint32)
    w0 = np.eye(4, dtype=np.uint32)
    w2 = np.array([[i + j + 1 for j in range(2)] for i in range(4)], np.uint32)
    rc, raw, _, _ = O.prove_gkr_chain(x, [("linear", w0), ("layernorm", None), ("linear", w2)], n_queries=5,
                                      v1_layout=True)
    assert rc == 0
    t = felts(raw)
    coms = t[1 + t[0]:]
    assert [hex(c) for c in coms[1:1 + coms[0]]] == GOLD["d10_weight_commitments"]


def test_layernorm_chain_runs():
    x = uniform_m31(4 * 32, 9).reshape(4, 32) % 3000
    w = (uniform_m31(32 * 16, 10).reshape(32, 16) % 7).astype(np.uint32)
    rc, raw, _, _ = O.prove_gkr_chain(x, [("layernorm", None), ("linear", w), ("layernorm", None)], n_queries=4)
    assert rc == 0
    assert felts(raw)[0] == 3 and felts(raw)[1] == 4
