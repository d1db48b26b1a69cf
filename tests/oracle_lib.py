"""ctypes binding of the CPU oracle (oracle/_build/liboracle.so).

Test infrastructure: imported only by tests/, __graft_entry__.smoke() and
bench.py's CPU legs, as the checker -- never by the product package.
"""
import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[1]
LIB_PATH = ROOT / "oracle" / "_build" / "liboracle.so"

u32p = np.ctypeslib.ndpointer(np.uint32, flags="C_CONTIGUOUS")
u64p = np.ctypeslib.ndpointer(np.uint64, flags="C_CONTIGUOUS")


class Channel(C.Structure):
    _fields_ = [("digest", C.c_uint64 * 4), ("n_draws", C.c_uint32), ("reserved", C.c_uint32),
                ("hash_count", C.c_uint64)]

    def digest_int(self) -> int:
        return sum(int(self.digest[i]) << (64 * i) for i in range(4))


def build() -> None:
    src = ROOT / "oracle" / "oracle.c"
    if not LIB_PATH.exists() or LIB_PATH.stat().st_mtime < src.stat().st_mtime:
        subprocess.run(["make", "-s", "-C", str(ROOT / "oracle")], check=True)


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        L = C.CDLL(str(LIB_PATH))
        chp = C.POINTER(Channel)
        sz = C.c_size_t
        L.orc_hades.argtypes = [u64p]
        L.orc_poseidon_hash.argtypes = [u64p, u64p, u64p]
        L.orc_poseidon_hash_many.argtypes = [u64p, sz, u64p]
        L.orc_felt_mul.argtypes = [u64p, u64p, u64p]
        L.orc_ch_init.argtypes = [chp]
        L.orc_ch_mix_u64.argtypes = [chp, C.c_uint64]
        L.orc_ch_mix_felt.argtypes = [chp, u64p]
        L.orc_ch_draw_felt.argtypes = [chp, u64p]
        L.orc_ch_draw_qm31.argtypes = [chp, u32p]
        L.orc_ch_mix_poly_coeffs.argtypes = [chp, u32p]
        L.orc_ch_mix_poly_coeffs_deg3.argtypes = [chp, u32p]
        L.orc_ch_mix_felts.argtypes = [chp, u32p, sz]
        L.orc_securefield_to_felt.argtypes = [u32p, u64p]
        L.orc_qm31_mul.argtypes = [u32p, u32p, u32p]
        L.orc_qm31_inv.argtypes = [u32p, u32p]
        L.orc_lagrange_basis.argtypes = [u32p, sz, u32p]
        L.orc_evaluate_mle.argtypes = [u32p, sz, u32p, u32p]
        L.orc_restrict_mle.argtypes = [u32p, sz, u32p, sz, u32p]
        L.orc_reduce_matmul_layer.argtypes = [u32p, sz, sz, u32p, sz, sz, u32p, sz, u32p, sz, sz, chp,
                                              u32p, u32p, u32p, u32p, C.c_int, C.c_int]
        L.orc_reduce_matmul_gkr.argtypes = [u32p, sz, u32p, u32p, sz, sz, u32p, sz, chp, u32p, u32p,
                                            u32p, u32p, C.c_int, C.c_int]
        L.orc_merkle_root_qm31.argtypes = [u32p, sz, u64p, C.c_int]
        L.orc_merkle_path_qm31.argtypes = [u32p, sz, sz, u64p, C.c_int]
        L.orc_merkle_verify.argtypes = [u64p, sz, u64p, u64p, sz]
        L.orc_prove_mle_opening.argtypes = [u32p, sz, u32p, chp, sz, u64p, u64p, sz, C.POINTER(sz),
                                            C.c_int]
        L.orc_verify_mle_opening.argtypes = [u64p, u64p, sz, u32p, sz, chp, sz, u32p]
        L.orc_prove_gkr_matmul.argtypes = [u32p, sz, sz, u32p, sz, C.c_void_p, sz, u64p, sz,
                                           C.POINTER(sz), u64p, u64p, C.c_int]
        L.orc_verify_gkr_matmul.argtypes = [u32p, sz, sz, u32p, sz, C.c_void_p, sz, u64p, sz, u64p]
        L.orc_io_commitment.argtypes = [u32p, sz, sz, u32p, sz, sz, u64p]
        L.orc_matmul_m31.argtypes = [u32p, sz, sz, u32p, sz, u32p, C.c_int]
        L.orc_activation_table.argtypes = [C.c_int, C.c_uint, u32p]
        L.orc_activation_table_log_size.argtypes = [C.c_int]
        L.orc_activation_table_log_size.restype = C.c_uint
        L.orc_reduce_activation_logup.argtypes = [u32p, sz, sz, C.c_int, u32p, sz, u32p, chp, u64p, sz,
                                                  C.POINTER(sz), u32p]
        L.orc_verify_activation_logup.argtypes = [u64p, sz, u32p, sz, u32p, chp, u32p]
        L.orc_weight_commitment.argtypes = [u32p, sz, sz, u64p, C.c_int]
        L.orc_prove_aggregated_binding.argtypes = [C.c_void_p, sz, chp, sz, u64p, sz, C.POINTER(sz), C.c_int]
        L.orc_verify_aggregated_binding.argtypes = [C.c_void_p, sz, u64p, sz, chp, sz]
        L.orc_activation_integer.argtypes = [C.c_int, C.c_uint32]
        L.orc_activation_integer.restype = C.c_uint32
        L.orc_piecewise_coeffs.argtypes = [C.c_int, u32p, u32p]
        L.orc_reduce_activation_piecewise.argtypes = [u32p, sz, sz, C.c_int, u32p, sz, u32p, chp, u64p, sz,
                                                      C.POINTER(sz), u32p, u32p]
        L.orc_verify_activation_piecewise.argtypes = [u64p, sz, u32p, sz, u32p, chp, u32p]
        L.orc_prove_gkr_chain.argtypes = [u32p, sz, sz, C.c_void_p, sz, C.c_void_p, sz, C.c_int, u64p, sz,
                                          C.POINTER(sz), u64p, u64p, C.c_int]
        L.orc_reduce_activation_relu.argtypes = [u32p, sz, sz, u32p, sz, u32p, chp, u64p, sz, C.POINTER(sz), u32p,
                                                 u32p]
        L.orc_rsqrt_table.argtypes = [C.c_uint, u32p]
        L.orc_reduce_rmsnorm.argtypes = [u32p, sz, sz, sz, C.c_void_p, sz, C.c_int, u32p, sz, u32p, chp, u64p,
                                         sz, C.POINTER(sz), u32p]
        L.orc_verify_rmsnorm.argtypes = [u64p, sz, sz, u32p, sz, u32p, chp, u32p]
        L.orc_reduce_layernorm.argtypes = [u32p, sz, sz, sz, u32p, sz, u32p, chp, u64p, sz, C.POINTER(sz), u32p]
        _lib = L
    return _lib


def threads() -> int:
    return int(os.environ.get("ORACLE_THREADS", os.cpu_count() or 1))


def felt(x: int) -> np.ndarray:
    return np.array([(x >> (64 * i)) & (2**64 - 1) for i in range(4)], dtype=np.uint64)


def felt_int(a) -> int:
    return sum(int(a[i]) << (64 * i) for i in range(4))


def new_channel() -> Channel:
    ch = Channel()
    lib().orc_ch_init(C.byref(ch))
    return ch


def poseidon_hash(a: int, b: int) -> int:
    out = np.zeros(4, np.uint64)
    lib().orc_poseidon_hash(felt(a), felt(b), out)
    return felt_int(out)


def poseidon_hash_many(xs) -> int:
    arr = np.concatenate([felt(x) for x in xs]) if xs else np.zeros(4, np.uint64)
    out = np.zeros(4, np.uint64)
    lib().orc_poseidon_hash_many(arr, len(xs), out)
    return felt_int(out)


def reduce_matmul_layer(a, b, r_i, r_j, ch, mode=1, nthreads=None):
    """a: (m,k) uint32, b: (k,n) uint32, r_i/r_j: (v,4) uint32. Returns dict."""
    a = np.ascontiguousarray(a, np.uint32)
    b = np.ascontiguousarray(b, np.uint32)
    m, k = a.shape
    _, n = b.shape
    pk = 1 << max(0, (k - 1).bit_length())
    log_k = pk.bit_length() - 1
    r_i = np.ascontiguousarray(r_i, np.uint32).reshape(-1, 4)
    r_j = np.ascontiguousarray(r_j, np.uint32).reshape(-1, 4)
    rp = np.zeros((max(log_k, 1), 12), np.uint32)
    chal = np.zeros((max(log_k, 1), 4), np.uint32)
    fa = np.zeros(4, np.uint32)
    fb = np.zeros(4, np.uint32)
    rc = lib().orc_reduce_matmul_layer(a.reshape(-1), m, k, b.reshape(-1), k, n,
                                       r_i.reshape(-1) if r_i.size else np.zeros(4, np.uint32),
                                       len(r_i), r_j.reshape(-1) if r_j.size else np.zeros(4, np.uint32),
                                       len(r_j), pk, C.byref(ch), rp.reshape(-1), chal.reshape(-1), fa, fb,
                                       mode, nthreads or threads())
    assert rc == 0, rc
    return {"round_polys": rp[:log_k], "challenges": chal[:log_k], "final_a": fa, "final_b": fb}


def merkle_root_qm31(evals, nthreads=None) -> int:
    e = np.ascontiguousarray(evals, np.uint32).reshape(-1)
    out = np.zeros(4, np.uint64)
    lib().orc_merkle_root_qm31(e, e.size // 4, out, nthreads or threads())
    return felt_int(out)


def prove_gkr_matmul(inp, w, policy=None, n_queries=10, cap=1 << 16):
    inp = np.ascontiguousarray(inp, np.uint32)
    w = np.ascontiguousarray(w, np.uint32)
    m, k = inp.shape
    _, n = w.shape
    buf = np.zeros(4 * cap, np.uint64)
    ln = C.c_size_t(0)
    dig = np.zeros(4, np.uint64)
    io = np.zeros(4, np.uint64)
    pol = None if policy is None else felt(policy).ctypes.data_as(C.c_void_p)
    pol_arr = None if policy is None else felt(policy)
    if pol_arr is not None:
        pol = pol_arr.ctypes.data_as(C.c_void_p)
    rc = lib().orc_prove_gkr_matmul(inp.reshape(-1), m, k, w.reshape(-1), n, pol, n_queries, buf, cap,
                                    C.byref(ln), dig, io, threads())
    assert rc == 0, rc
    cd = [felt_int(buf[4 * i:4 * i + 4]) for i in range(ln.value)]
    return {"calldata": cd, "digest": felt_int(dig), "io": felt_int(io), "raw": buf[:4 * ln.value].copy()}


def verify_gkr_matmul(inp, w, raw, policy=None, n_queries=10):
    inp = np.ascontiguousarray(inp, np.uint32)
    w = np.ascontiguousarray(w, np.uint32)
    m, k = inp.shape
    _, n = w.shape
    dig = np.zeros(4, np.uint64)
    pol_arr = None if policy is None else felt(policy)
    pol = None if pol_arr is None else pol_arr.ctypes.data_as(C.c_void_p)
    ok = lib().orc_verify_gkr_matmul(inp.reshape(-1), m, k, w.reshape(-1), n, pol, n_queries,
                                     np.ascontiguousarray(raw, np.uint64), raw.size // 4, dig)
    return bool(ok), felt_int(dig)


def reduce_activation_logup(inp, tag, point, value, ch, cap=1 << 22):
    inp = np.ascontiguousarray(inp, np.uint32)
    rows, cols = inp.shape
    point = np.ascontiguousarray(point, np.uint32).reshape(-1, 4)
    buf = np.zeros(4 * cap, np.uint64)
    ln = C.c_size_t(0)
    ie = np.zeros(4, np.uint32)
    rc = lib().orc_reduce_activation_logup(inp.reshape(-1), rows, cols, tag, point.reshape(-1), len(point),
                                           np.ascontiguousarray(value, np.uint32), C.byref(ch), buf, cap,
                                           C.byref(ln), ie)
    return rc, buf[:4 * ln.value].copy(), ie


def verify_activation_logup(raw, point, value, ch):
    point = np.ascontiguousarray(point, np.uint32).reshape(-1, 4)
    ie = np.zeros(4, np.uint32)
    ok = lib().orc_verify_activation_logup(np.ascontiguousarray(raw, np.uint64), raw.size // 4, point.reshape(-1),
                                           len(point), np.ascontiguousarray(value, np.uint32), C.byref(ch), ie)
    return bool(ok), ie


def rsqrt_table(log_size: int = 16) -> np.ndarray:
    t = np.zeros(1 << log_size, np.uint32)
    assert lib().orc_rsqrt_table(log_size, t) == 0
    return t


def reduce_rmsnorm(inp, dim, point, value, ch, gamma=None, skip_rms_sq=False, cap=1 << 18):
    inp = np.ascontiguousarray(inp, np.uint32)
    rows, cols = inp.shape
    point = np.ascontiguousarray(point, np.uint32).reshape(-1, 4)
    g = None if gamma is None else np.ascontiguousarray(gamma, np.uint32)
    buf = np.zeros(4 * cap, np.uint64)
    ln = C.c_size_t(0)
    ie = np.zeros(4, np.uint32)
    rc = lib().orc_reduce_rmsnorm(inp.reshape(-1), rows, cols, dim,
                                  None if g is None else g.ctypes.data_as(C.c_void_p), 0 if g is None else g.size,
                                  int(skip_rms_sq), point.reshape(-1), len(point),
                                  np.ascontiguousarray(value, np.uint32), C.byref(ch), buf, cap, C.byref(ln), ie)
    return rc, buf[:4 * ln.value].copy(), ie


def reduce_layernorm(inp, dim, point, value, ch, cap=1 << 18):
    inp = np.ascontiguousarray(inp, np.uint32)
    rows, cols = inp.shape
    point = np.ascontiguousarray(point, np.uint32).reshape(-1, 4)
    buf = np.zeros(4 * cap, np.uint64)
    ln = C.c_size_t(0)
    ie = np.zeros(4, np.uint32)
    rc = lib().orc_reduce_layernorm(inp.reshape(-1), rows, cols, dim, point.reshape(-1), len(point),
                                    np.ascontiguousarray(value, np.uint32), C.byref(ch), buf, cap, C.byref(ln), ie)
    return rc, buf[:4 * ln.value].copy(), ie


def verify_rmsnorm(raw, dim, point, value, ch):
    point = np.ascontiguousarray(point, np.uint32).reshape(-1, 4)
    ie = np.zeros(4, np.uint32)
    ok = lib().orc_verify_rmsnorm(np.ascontiguousarray(raw, np.uint64), raw.size // 4, dim, point.reshape(-1),
                                  len(point), np.ascontiguousarray(value, np.uint32), C.byref(ch), ie)
    return bool(ok), ie


def rmsnorm_output_eval(raw) -> np.ndarray:
    """output_eval of a LayerProof::RMSNorm record (felts 5..8)."""
    return np.array([raw[4 * (5 + i)] for i in range(4)], np.uint32)


class WeightClaim(C.Structure):
    _fields_ = [("weight", C.c_void_p), ("rows", C.c_size_t), ("cols", C.c_size_t),
                ("matrix_index", C.c_size_t), ("eval_point", C.c_void_p),
                ("expected_value", C.c_uint32 * 4), ("commitment", C.c_uint64 * 4)]


def weight_commitment(w) -> np.ndarray:
    w = np.ascontiguousarray(w, np.uint32)
    out = np.zeros(4, np.uint64)
    lib().orc_weight_commitment(w.reshape(-1), w.shape[0], w.shape[1], out, threads())
    return out


def make_claims(specs):
    """specs: list of (weight matrix, matrix_index, eval_point (n, 4), value (4,), commitment (4,) u64).
    Returns the ctypes array and the arrays it points into (keep both alive)."""
    keep = []
    arr = (WeightClaim * len(specs))()
    for i, (w, idx, pt, val, com) in enumerate(specs):
        w = np.ascontiguousarray(w, np.uint32)
        pt = np.ascontiguousarray(pt, np.uint32).reshape(-1)
        keep += [w, pt]
        arr[i].weight = w.ctypes.data
        arr[i].rows, arr[i].cols = w.shape
        arr[i].matrix_index = idx
        arr[i].eval_point = pt.ctypes.data if pt.size else None
        for j in range(4):
            arr[i].expected_value[j] = int(val[j])
            arr[i].commitment[j] = int(com[j])
    return arr, keep


def prove_aggregated_binding(specs, ch, n_queries=10, cap=1 << 20):
    arr, keep = make_claims(specs)
    buf = np.zeros(4 * cap, np.uint64)
    ln = C.c_size_t(0)
    rc = lib().orc_prove_aggregated_binding(C.cast(arr, C.c_void_p), len(specs), C.byref(ch), n_queries, buf, cap,
                                            C.byref(ln), threads())
    return rc, buf[:4 * ln.value].copy()


def verify_aggregated_binding(specs, raw, ch, n_queries=10):
    arr, keep = make_claims(specs)
    return bool(lib().orc_verify_aggregated_binding(C.cast(arr, C.c_void_p), len(specs),
                                                    np.ascontiguousarray(raw, np.uint64), raw.size // 4,
                                                    C.byref(ch), n_queries))


def mle_col_major(w) -> np.ndarray:
    """matrix_to_mle_col_major_padded as (n, 4) QM31 words."""
    rows, cols = w.shape
    pr, pc = 1 << max(0, (rows - 1).bit_length()), 1 << max(0, (cols - 1).bit_length())
    v = np.zeros((pc, pr), np.uint32)
    v[:cols, :rows] = np.asarray(w, np.uint32).T % np.uint32((1 << 31) - 1)
    out = np.zeros((pr * pc, 4), np.uint32)
    out[:, 0] = v.reshape(-1)
    return out


def evaluate_mle(evals, point) -> np.ndarray:
    evals = np.ascontiguousarray(evals, np.uint32).reshape(-1, 4)
    point = np.ascontiguousarray(point, np.uint32).reshape(-1, 4)
    out = np.zeros(4, np.uint32)
    lib().orc_evaluate_mle(evals.reshape(-1), len(point), point.reshape(-1), out)
    return out


def restrict_mle(evals, assign) -> np.ndarray:
    """restrict_mle (backend.rs:199-215): fix the first len(assign) variables."""
    evals = np.ascontiguousarray(evals, np.uint32).reshape(-1, 4)
    assign = np.ascontiguousarray(assign, np.uint32).reshape(-1, 4)
    out = np.zeros((len(evals) >> len(assign), 4), np.uint32)
    lib().orc_restrict_mle(evals.reshape(-1), len(evals), assign.reshape(-1), len(assign), out.reshape(-1))
    return out


def piecewise_coeffs(tag):
    sl, ic = np.zeros(16, np.uint32), np.zeros(16, np.uint32)
    assert lib().orc_piecewise_coeffs(tag, sl, ic) == 0
    return sl, ic


def reduce_activation_piecewise(inp, tag, point, value, ch, cap=1 << 16):
    inp = np.ascontiguousarray(inp, np.uint32)
    rows, cols = inp.shape
    point = np.ascontiguousarray(point, np.uint32).reshape(-1, 4)
    buf = np.zeros(4 * cap, np.uint64)
    ln = C.c_size_t(0)
    ie = np.zeros(4, np.uint32)
    nxt = np.zeros((len(point), 4), np.uint32)
    rc = lib().orc_reduce_activation_piecewise(inp.reshape(-1), rows, cols, tag, point.reshape(-1), len(point),
                                               np.ascontiguousarray(value, np.uint32), C.byref(ch), buf, cap,
                                               C.byref(ln), ie, nxt.reshape(-1))
    nv = (rows - 1).bit_length() + (cols - 1).bit_length()
    return rc, buf[:4 * ln.value].copy(), ie, nxt[:nv].copy()


def verify_activation_piecewise(raw, point, value, ch):
    point = np.ascontiguousarray(point, np.uint32).reshape(-1, 4)
    ie = np.zeros(4, np.uint32)
    ok = lib().orc_verify_activation_piecewise(np.ascontiguousarray(raw, np.uint64), raw.size // 4,
                                               point.reshape(-1), len(point), np.ascontiguousarray(value, np.uint32),
                                               C.byref(ch), ie)
    return bool(ok), ie


class ChainLayer(C.Structure):
    _fields_ = [("type", C.c_int), ("weight", C.c_void_p), ("n", C.c_size_t), ("src", C.c_longlong),
                ("lhs", C.c_longlong)]


CHAIN_PREV = -2
_CHAIN_KINDS = {"linear": 0, "relu": 1, "rmsnorm": 2, "add": 3, "mul": 4, "layernorm": 5, "activation": 6}
_ACT_TAGS = {"gelu": 2, "sigmoid": 3, "softmax": 4, "silu": 5}


def chain_layers(layers):
    """ctypes array for layers given as (kind, arg[, src]): ("linear", weight (rows, n)),
    ("relu", None), ("rmsnorm", None), ("layernorm", None), ("add", lhs layer), ("mul", lhs layer); src is the
    layer feeding this one (None = the previous layer, -1 = the model input)."""
    keep = []
    arr = (ChainLayer * len(layers))()
    for i, spec in enumerate(layers):
        kind, arg = spec[0], spec[1]
        src = spec[2] if len(spec) > 2 and spec[2] is not None else CHAIN_PREV
        arr[i].type, arr[i].weight, arr[i].n, arr[i].src, arr[i].lhs = _CHAIN_KINDS[kind], None, 0, src, -1
        if kind == "linear":
            w = np.ascontiguousarray(arg, np.uint32)
            keep.append(w)
            arr[i].weight, arr[i].n = w.ctypes.data, w.shape[1]
        elif kind in ("add", "mul"):
            arr[i].lhs = int(arg)
        elif kind == "activation":
            arr[i].n = _ACT_TAGS[arg.lower()] if isinstance(arg, str) else int(arg)
    return arr, keep


def prove_gkr_chain(inp, layers, n_queries=10, policy=None, legacy_layout=False, v1_layout=False, cap=1 << 20,
                    activation_logup=False):
    """layers: see chain_layers.  v1_layout: the verify_model_gkr calldata from proof_data on."""
    inp = np.ascontiguousarray(inp, np.uint32)
    m, k0 = inp.shape
    arr, keep = chain_layers(layers)
    buf = np.zeros(4 * cap, np.uint64)
    ln = C.c_size_t(0)
    dig = np.zeros(4, np.uint64)
    io = np.zeros(4, np.uint64)
    pol = None if policy is None else felt(policy)
    rc = lib().orc_prove_gkr_chain(inp.reshape(-1), m, k0, C.cast(arr, C.c_void_p), len(layers),
                                   None if pol is None else pol.ctypes.data_as(C.c_void_p), n_queries,
                                   int(legacy_layout) | (2 if v1_layout else 0) | (4 if activation_logup else 0),
                                   buf, cap,
                                   C.byref(ln), dig, io, threads())
    return rc, buf[:4 * ln.value].copy(), felt_int(dig), felt_int(io)


def verify_gkr_chain(inp, layers, raw, n_queries=10, policy=None, activation_logup=False):
    """orc_verify_gkr_chain on a serialize_gkr_model_proof of a Linear / Activation / RMSNorm
    chain: (accepted, verifier digest)."""
    inp = np.ascontiguousarray(inp, np.uint32)
    m, k0 = inp.shape
    arr, keep = chain_layers(layers)
    raw = np.ascontiguousarray(raw, np.uint64)
    dig = np.zeros(4, np.uint64)
    pol = None if policy is None else felt(policy)
    L = lib()
    L.orc_verify_gkr_chain.argtypes = [u32p, C.c_size_t, C.c_size_t, C.c_void_p, C.c_size_t, C.c_void_p, C.c_size_t,
                                       C.c_int, u64p, C.c_size_t, u64p, C.c_int]
    ok = L.orc_verify_gkr_chain(inp.reshape(-1), m, k0, C.cast(arr, C.c_void_p), len(layers),
                                None if pol is None else pol.ctypes.data_as(C.c_void_p), n_queries,
                                4 if activation_logup else 0, raw, raw.size // 4, dig, threads())
    return bool(ok), felt_int(dig)


def reduce_activation_relu(inp, point, value, ch, cap=1 << 14):
    inp = np.ascontiguousarray(inp, np.uint32)
    rows, cols = inp.shape
    point = np.ascontiguousarray(point, np.uint32).reshape(-1, 4)
    buf = np.zeros(4 * cap, np.uint64)
    ln = C.c_size_t(0)
    ie = np.zeros(4, np.uint32)
    nxt = np.zeros((max(len(point), 1), 4), np.uint32)
    rc = lib().orc_reduce_activation_relu(inp.reshape(-1), rows, cols, point.reshape(-1), len(point),
                                          np.ascontiguousarray(value, np.uint32), C.byref(ch), buf, cap, C.byref(ln),
                                          ie, nxt.reshape(-1))
    nv = (rows - 1).bit_length() + (cols - 1).bit_length()
    return rc, buf[:4 * ln.value].copy(), ie, nxt[:nv].copy()
