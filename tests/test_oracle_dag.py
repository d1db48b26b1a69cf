"""The oracle's DAG circuits (Add / Mul layers with deferred skip-branch proofs) and the
verify_model_gkr calldata layout, pinned against the reference's artifacts:

* d9_verify_gkr_calldata.txt (sp3_mlp model, model id 0xd9): every felt of the V1 calldata,
  after removing the Activation record's trailing piecewise flag, which the artifact predates;
* d11 (Linear -> fork -> ReLU -> Linear -> add_from(fork)): the Add record, the first
  round of the next MatMul sumcheck, the io commitment and the weight commitments.
"""
import json
from pathlib import Path

import numpy as np
import pytest

import oracle_lib as O
from helpers import int_matrix_m31

GOLD = json.loads((Path(__file__).parent / "golden" / "reference_vectors.json").read_text())
P = (1 << 31) - 1


def felts(raw):
    b = raw.reshape(-1, 4)
    return [sum(int(r[i]) << (64 * i) for i in range(4)) for r in b]


def v1_envelope(model_id, x, y, layers, n_proofs):
    """verify_model_gkr's leading arguments (starknet.rs:3168-3200) for a chain proof."""
    m, k0 = x.shape
    out = [model_id, 6 + x.size + y.size, m, k0, x.size, *map(int, x.reshape(-1)), y.shape[0], y.shape[1], y.size,
           *map(int, y.reshape(-1)), len(layers), n_proofs]
    widths, dims = [k0], []
    for spec in layers:
        widths.append(spec[1].shape[1] if spec[0] == "linear" else widths[-1])
    for i in reversed(range(len(layers))):
        if layers[i][0] == "linear":
            dims += [m, widths[i], widths[i + 1]]
    return out + [len(dims), *dims, 0]


def sp3_model():
    g = GOLD["sp3_mlp"]
    x = np.array([g["input"]], np.uint32)
    w0, w2 = (np.array(w, np.uint32) for w in g["weights"])
    return x, [("linear", w0), ("relu", None), ("linear", w2)], np.array([g["output"]], np.uint32)


def drop_piecewise_flag(tail, relu_at=26, walk_tail=26 + 1):
    """The V1 tail without the ReLU record's last felt (its piecewise flag); the ReLU record sits
    between the first MatMul record (26 felts) and the last MatMul record + deferred count."""
    pd_len = tail[0]
    idx = 1 + pd_len - walk_tail - 1
    assert tail[idx] == 0
    return [pd_len - 1] + tail[1:idx] + tail[idx + 1:]


def test_d9_verify_calldata_reproduced():
    g = GOLD["d9_verify_calldata"]
    x, layers, y = sp3_model()
    rc, raw, dig, io = O.prove_gkr_chain(x, layers, n_queries=g["n_queries"], v1_layout=True)
    assert rc == 0
    tail = drop_piecewise_flag(felts(raw))
    mine = v1_envelope(int(g["model_id"], 16), x, y, layers, 3) + tail
    assert mine == [int(h, 16) for h in g["calldata"]]


def d11_model():
    g = GOLD["d11_residual"]
    x = np.array(g["input"], np.uint32)
    w0, w2 = np.array(g["w0"], np.uint32), np.array(g["w2"], np.uint32)
    return x, [("linear", w0), ("relu", None), ("linear", w2), ("add", 0)]


def test_d11_residual_pins():
    g = GOLD["d11_residual"]
    x, layers = d11_model()
    rc, raw, dig, io = O.prove_gkr_chain(x, layers, n_queries=5, v1_layout=True)
    assert rc == 0
    tail = felts(raw)
    pd = tail[1:1 + tail[0]]
    assert pd[:10] == g["add_record"]
    assert pd[10:12] == [0, 2]  # MatMul tag, 2 rounds
    assert pd[12:16] == g["matmul_round0_c0"] and pd[16:20] == g["matmul_round0_c2"]
    assert io == int(g["io_commitment"], 16)
    coms = tail[1 + tail[0]:]
    assert coms[0] == 3  # the walk's two weights, then the deferred branch's (W0 again)
    assert coms[1:3] == [int(c, 16) for c in g["weight_commitments"]] and coms[3] == coms[2]
    # the deferred record: count 1, the skip claim (the Add's lhs), kind MatMul, m k n
    dstart = len(pd) - (4 + 1 + 3 + 1 + 2 * 8 + 8 + 1) - 1
    assert pd[dstart] == 1 and pd[dstart + 1:dstart + 5] == g["add_record"][1:5]
    assert pd[dstart + 5:dstart + 9] == [0, 1, 4, 4]


def test_model_proof_layout_omits_deferred():
    x, layers = d11_model()
    rc, raw, _, io = O.prove_gkr_chain(x, layers, n_queries=5)
    assert rc == 0
    f = felts(raw)
    assert f[0] == 4 and f[1:11] == GOLD["d11_residual"]["add_record"]
    assert f[-1] == io


def mul_circuit(seed, m=2, d=8, e=4):
    x = int_matrix_m31(m, d, seed, bound=30)
    return x, [("linear", int_matrix_m31(d, 2 * d, seed + 1, bound=9)),      # 0: gate branch
               ("linear", int_matrix_m31(2 * d, 2 * d, seed + 2, bound=9)),  # 1
               ("relu", None),                                              # 2
               ("mul", 0),                                                  # 3: lhs = layer 0
               ("linear", int_matrix_m31(2 * d, e, seed + 3, bound=9))]     # 4


def test_mul_circuit_structure():
    x, layers = mul_circuit(3)
    rc, raw, _, _ = O.prove_gkr_chain(x, layers, n_queries=4, v1_layout=True)
    assert rc == 0
    tail = felts(raw)
    pd = tail[1:1 + tail[0]]
    # walk: Linear 4, Mul 3 (skips layer 0), ReLU 2, Linear 1; then one deferred MatMul (layer 0)
    nv = 1 + 4  # log2(2) + log2(16)
    assert pd[0] == 0
    off = 2 + 8 * 4 + 8  # after Linear 4's record (k = 16: 4 rounds)
    assert pd[off] == 2 and pd[off + 1] == nv
    rc2, raw2, _, _ = O.prove_gkr_chain(x, layers, n_queries=4)
    f = felts(raw2)
    assert f[0] == 4  # four layer records: the skipped layer has none
    assert tail[1 + tail[0]] == 3  # commitments: Linear 4, Linear 1, deferred Linear 0


def test_deferred_branch_must_be_linear():
    x = int_matrix_m31(2, 8, 5, bound=30)
    layers = [("linear", int_matrix_m31(8, 8, 6, bound=9)), ("relu", None),
              ("linear", int_matrix_m31(8, 8, 7, bound=9)), ("mul", 1)]
    rc, _, _, _ = O.prove_gkr_chain(x, layers, n_queries=4)
    assert rc == 4


def test_bad_dag_rejected():
    x = int_matrix_m31(2, 8, 5, bound=30)
    w = int_matrix_m31(8, 4, 6, bound=9)
    assert O.prove_gkr_chain(x, [("linear", w), ("add", 1)], n_queries=4)[0] == 1  # lhs must be lower
    assert O.prove_gkr_chain(x, [("linear", w), ("relu", None), ("add", 0, -1)], n_queries=4)[0] == 1  # widths


def test_d7_verify_calldata_reproduced():
    g = GOLD["d7_verify_calldata"]
    a = GOLD["sp3_matmul_only"]
    x = np.array([[1, 2, 3, 4]], np.uint32)
    w = np.array([[2 * i + j + 1 for j in range(2)] for i in range(4)], np.uint32)
    rc, raw, _, io = O.prove_gkr_chain(x, [("linear", w)], n_queries=10, v1_layout=True)
    assert rc == 0
    mine = v1_envelope(int(g["model_id"], 16), x, np.array([[50, 60]], np.uint32), [("linear", w)], 1) + felts(raw)
    assert mine == [int(h, 16) for h in g["calldata"]]
    assert io == int(a["io_commitment"], 16)


@pytest.mark.parametrize("name", ["d7", "d9", "d11"])
def test_register_calldata(name):
    import zkml_b200 as Z
    ref = GOLD["register_calldata"][name]
    if name == "d7":
        layers = [("linear", None)]
    elif name == "d9":
        layers = sp3_model()[1]
    else:
        layers = d11_model()[1]
    coms = [int(c, 16) for c in ref[2:2 + int(ref[1])]]
    assert Z.build_register_gkr_calldata(int(ref[0], 16), coms, layers) == ref


@pytest.mark.parametrize("name", ["d9", "d11"])
def test_register_calldata_from_proof_commitments(name):
    """register_model_gkr calldata from the weight commitments of an oracle-built verify calldata."""
    import zkml_b200 as Z
    ref = GOLD["register_calldata"][name]
    if name == "d9":
        x, layers, y = sp3_model()
    else:
        x, layers = d11_model()
        y = np.array([[19, 21, 26, 22]], np.uint32)
    rc, raw, _, _ = O.prove_gkr_chain(x, layers, n_queries=5, v1_layout=True)
    assert rc == 0
    tail = felts(raw)
    n_proofs = 3 if name == "d9" else 4
    cd = v1_envelope(int(ref[0], 16), x, y, layers, n_proofs) + tail
    coms = Z.verify_calldata_weight_commitments(cd, layers)
    assert Z.build_register_gkr_calldata(int(ref[0], 16), coms, layers) == ref


# --- verifier-side replay of the Add and Mul records (gkr/verifier.rs Add / Mul arms) --------------

def _cm(a, b):  # CM31 product, i^2 = -1
    return ((a[0] * b[0] - a[1] * b[1]) % P, (a[0] * b[1] + a[1] * b[0]) % P)


def qmul(x, y):
    """QM31 product: (a + b u)(c + d u) with u^2 = 2 + i."""
    a, b, c, d = (x[0], x[1]), (x[2], x[3]), (y[0], y[1]), (y[2], y[3])
    ac, bd = _cm(a, c), _cm(b, d)
    bdu = _cm(bd, (2, 1))
    ad, bc = _cm(a, d), _cm(b, c)
    return [(ac[0] + bdu[0]) % P, (ac[1] + bdu[1]) % P, (ad[0] + bc[0]) % P, (ad[1] + bc[1]) % P]


def qadd(x, y):
    return [(u + v) % P for u, v in zip(x, y)]


def qsub(x, y):
    return [(u - v) % P for u, v in zip(x, y)]


def mle_point_eval(vals, point):
    """MLE of M31 values (index bit n-1 = the first variable) at a QM31 point."""
    cur = [[int(v) % P, 0, 0, 0] for v in vals]
    for r in point:
        h = len(cur) // 2
        cur = [qadd(cur[i], qmul(r, qsub(cur[h + i], cur[i]))) for i in range(h)]
    return cur[0]


def test_add_and_mul_records_verify():
    """Replays the transcript up to a Mul record and checks the degree-3 eq-sumcheck the way the
    reference verifier does: c1 from the running claim, the final claim = eq(r, s) lhs(s) rhs(s);
    then the Add record: lhs + rhs equals the claim on its output."""
    import zkml_b200 as Z
    m, d = 2, 8
    x = int_matrix_m31(m, d, 21, bound=30)
    wa, wb = int_matrix_m31(d, d, 22, bound=9), int_matrix_m31(d, d, 23, bound=9)
    layers = [("linear", wa), ("linear", wb, -1), ("mul", 0), ("add", 1)]
    rc, raw, dig, io = O.prove_gkr_chain(x, layers, n_queries=4)
    assert rc == 0
    f = felts(raw)
    ya = (x.astype(object) @ wa.astype(object)) % P
    yb = (x.astype(object) @ wb.astype(object)) % P
    ymul = (ya * yb) % P
    yout = (ymul + yb) % P
    nv = (m - 1).bit_length() + (d - 1).bit_length()
    ch = Z.PoseidonChannel()
    for v in (4, m, d):
        ch.mix_u64(v)
    point = [list(map(int, ch.draw_qm31())) for _ in range(nv)]
    claim = mle_point_eval(yout.reshape(-1), point)
    ch.mix_felt(Z.securefield_to_felt(np.array(claim, np.uint32)))
    # Add record (walk starts at layer 3): tag, lhs, rhs, trunk
    assert f[1] == 1
    lhs, rhs = f[2:6], f[6:10]
    assert qadd(lhs, rhs) == claim
    assert lhs == mle_point_eval(yb.reshape(-1), point) and rhs == mle_point_eval(ymul.reshape(-1), point)
    assert f[10] == 1  # rhs (layer 2) is the trunk
    ch.mix_felt(Z.securefield_to_felt(np.array(lhs, np.uint32)))
    ch.mix_felt(Z.securefield_to_felt(np.array(rhs, np.uint32)))
    ch.draw_qm31()
    claim = rhs
    # Mul record: tag 2, rounds, (c0, c2, c3) per round, lhs, rhs
    at = 11
    assert f[at] == 2 and f[at + 1] == nv
    ch.mix_u64(0x4D554C)
    ch.mix_felt(Z.securefield_to_felt(np.array(claim, np.uint32)))
    cur, chal = claim, []
    for r in range(nv):
        base = at + 2 + 12 * r
        c0, c2, c3 = f[base:base + 4], f[base + 4:base + 8], f[base + 8:base + 12]
        c1 = qsub(qsub(qsub(cur, qadd(c0, c0)), c2), c3)
        ch.mix_poly_coeffs_deg3(*(np.array(c, np.uint32) for c in (c0, c1, c2, c3)))
        s = list(map(int, ch.draw_qm31()))
        chal.append(s)
        cur = qadd(qadd(c0, qmul(c1, s)), qmul(qadd(c2, qmul(c3, s)), qmul(s, s)))
    ml, mr = f[at + 2 + 12 * nv:at + 6 + 12 * nv], f[at + 6 + 12 * nv:at + 10 + 12 * nv]
    eq = [1, 0, 0, 0]
    for r, s in zip(point, chal):
        one_r, one_s = qsub([1, 0, 0, 0], r), qsub([1, 0, 0, 0], s)
        eq = qmul(eq, qadd(qmul(r, s), qmul(one_r, one_s)))
    assert cur == qmul(qmul(eq, ml), mr)
    assert ml == mle_point_eval(ya.reshape(-1), chal) and mr == mle_point_eval(yb.reshape(-1), chal)
