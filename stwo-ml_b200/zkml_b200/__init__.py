"""B200-native GKR matmul-sumcheck prover: Python host interface.

Mirrors the stwo-ml engine's interface for this path so code written against
the reference reads the same:

* ``PoseidonChannel``      -- engine/src/crypto/poseidon_channel.rs:83-306
* ``M31Matrix``            -- engine/src/components/matmul.rs:85-116
* ``GpuBackend``           -- the ``ZkmlOps`` trait (engine/src/backend.rs:85-107):
  ``reduce_matmul_layer``, ``evaluate_mle_at_point``, ``restrict_mle``
* ``MatMulReduction``      -- backend.rs:73-79
* ``reduce_matmul_layer_with_backend`` -- engine/src/gkr/prover.rs:5959-6073
* ``prove_gkr_matmul`` / ``commit_mle_root`` / ``prove_mle_opening`` -- the
  single-layer GKR proof, Merkle commitment and weight opening
  (gkr/prover.rs:1500-2251, crypto/poseidon_merkle.rs, crypto/mle_opening.rs).

All compute runs in ``lib/libzkml_b200.so`` (CUDA, sm_100a) through its C ABI
(``include/zkml_b200.h``).  There is no CPU fallback: if the library or the
GPU is missing, the calls raise.

QM31 values are numpy ``uint32`` arrays of shape ``(..., 4)`` holding
``[a, b, c, d] = (a + b i) + (c + d i) u``; felt252 values are Python ints.
Matrix inputs may be numpy arrays (host) or CUDA torch tensors on the
context's device (used in place).
"""
from __future__ import annotations

import collections.abc as _abc
import ctypes as C
import os
import threading
from dataclasses import dataclass, field
from pathlib import Path
from typing import List, Optional, Sequence, Tuple

import numpy as np

_PKG = Path(__file__).resolve().parent
LIB_PATH = _PKG.parent / "lib" / "libzkml_b200.so"

M31_P = (1 << 31) - 1
STARK_P = 2**251 + 17 * 2**192 + 1

ZKML_OK = 0
_STATUS = {1: "INVALID_ARG", 2: "OOM", 3: "CUDA", 4: "NCCL", 5: "TIMEOUT", 6: "UNSUPPORTED", 7: "VERIFY"}


class ZkmlError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"zkml {_STATUS.get(status, status)}: {msg}")
        self.status = status


class InvalidArgument(ZkmlError, ValueError):
    pass


class _Channel(C.Structure):
    _fields_ = [("digest", C.c_uint64 * 4), ("n_draws", C.c_uint32), ("reserved", C.c_uint32),
                ("hash_count", C.c_uint64)]


_u32 = np.ctypeslib.ndpointer(np.uint32, flags="C_CONTIGUOUS")
_u64 = np.ctypeslib.ndpointer(np.uint64, flags="C_CONTIGUOUS")
_lib = None
_lib_lock = threading.Lock()

# Every symbol include/zkml_b200.h declares, with (restype, argtypes).
_SIGS = {
    "zkml_abi_version": (C.c_int, []),
    "zkml_last_error": (C.c_char_p, []),
    "zkml_ctx_create": (C.c_int, [C.c_int, C.POINTER(C.c_void_p)]),
    "zkml_ctx_destroy": (C.c_int, [C.c_void_p]),
    "zkml_ctx_device": (C.c_int, [C.c_void_p]),
    "zkml_ctx_kernel_launches": (C.c_uint64, [C.c_void_p]),
    "zkml_ctx_h2d_bytes": (C.c_uint64, [C.c_void_p]),
    "zkml_ctx_set_stream": (C.c_int, [C.c_void_p, C.c_void_p]),
    "zkml_ctx_enable_timing": (C.c_int, [C.c_void_p, C.c_int]),
    "zkml_ctx_kernel_time": (C.c_int, [C.c_void_p, C.c_char_p, C.POINTER(C.c_double), C.POINTER(C.c_uint64)]),
    "zkml_channel_init": (None, [C.POINTER(_Channel)]),
    "zkml_channel_mix_u64": (None, [C.POINTER(_Channel), C.c_uint64]),
    "zkml_channel_mix_felt": (None, [C.POINTER(_Channel), _u64]),
    "zkml_channel_mix_qm31": (None, [C.POINTER(_Channel), _u32]),
    "zkml_channel_draw_felt252": (None, [C.POINTER(_Channel), _u64]),
    "zkml_channel_draw_qm31": (None, [C.POINTER(_Channel), _u32]),
    "zkml_channel_mix_poly_coeffs": (None, [C.POINTER(_Channel), _u32]),
    "zkml_channel_mix_poly_coeffs_deg3": (None, [C.POINTER(_Channel), _u32]),
    "zkml_channel_mix_felts": (None, [C.POINTER(_Channel), _u32, C.c_size_t]),
    "zkml_hades_permutation": (None, [_u64]),
    "zkml_poseidon_hash": (None, [_u64, _u64, _u64]),
    "zkml_poseidon_hash_many": (None, [_u64, C.c_size_t, _u64]),
    "zkml_securefield_to_felt": (None, [_u32, _u64]),
    "zkml_reduce_matmul_layer": (C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t, C.c_size_t, C.c_void_p,
                                           C.c_size_t, C.c_size_t, C.c_void_p, C.c_size_t, C.c_void_p,
                                           C.c_size_t, C.c_size_t, C.POINTER(_Channel), _u32, _u32, _u32,
                                           _u32]),
    "zkml_evaluate_mle": (C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t, C.c_void_p, _u32]),
    "zkml_restrict_mle": (C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t, C.c_void_p, C.c_size_t, _u32]),
    "zkml_reduce_matmul_layer_gkr": (C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t, _u32, C.c_void_p,
                                               C.c_size_t, C.c_size_t, C.c_void_p, C.c_size_t,
                                               C.POINTER(_Channel), _u32, _u32, _u32, _u32]),
    "zkml_commit_mle_root": (C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t, _u64]),
    "zkml_prove_mle_opening": (C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t, C.c_void_p, C.POINTER(_Channel),
                                         C.c_size_t, _u64, _u64, C.c_size_t, C.POINTER(C.c_size_t)]),
    "zkml_io_commitment": (C.c_int, [_u32, C.c_size_t, C.c_size_t, _u32, C.c_size_t, C.c_size_t, _u64]),
    "zkml_activation_table": (C.c_int, [C.c_int, _u32, C.c_size_t, C.POINTER(C.c_size_t)]),
    "zkml_reduce_activation_logup": (C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t, C.c_size_t, C.c_int,
                                               C.c_void_p, C.c_size_t, _u32, C.POINTER(_Channel), _u64,
                                               C.c_size_t, C.POINTER(C.c_size_t), _u32]),
    "zkml_reduce_rmsnorm": (C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t, C.c_size_t, C.c_size_t, C.c_void_p,
                                      C.c_size_t, C.c_void_p, C.c_size_t, _u32, C.POINTER(_Channel), _u64,
                                      C.c_size_t, C.POINTER(C.c_size_t), _u32]),
    "zkml_reduce_layernorm": (C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t, C.c_size_t, C.c_size_t, C.c_void_p,
                                        C.c_size_t, _u32, C.POINTER(_Channel), _u64, C.c_size_t,
                                        C.POINTER(C.c_size_t), _u32]),
    "zkml_reduce_activation_piecewise": (C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t, C.c_size_t, C.c_int,
                                                   C.c_void_p, C.c_size_t, _u32, C.POINTER(_Channel), _u64,
                                                   C.c_size_t, C.POINTER(C.c_size_t), _u32, _u32]),
    "zkml_restrict_cols_block": (C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t, C.c_size_t, C.c_size_t, C.c_void_p,
                                           C.c_size_t, C.c_void_p]),
    "zkml_reduce_matmul_layer_gkr_fb": (C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t, _u32, C.c_void_p, C.c_size_t,
                                                  C.c_size_t, C.c_void_p, C.c_size_t, C.POINTER(_Channel), _u32,
                                                  _u32, _u32, _u32]),
    "zkml_reduce_activation_relu": (C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t, C.c_size_t, C.c_void_p,
                                              C.c_size_t, _u32, C.POINTER(_Channel), _u64, C.c_size_t,
                                              C.POINTER(C.c_size_t), _u32, _u32]),
    "zkml_prove_gkr_chain": (C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t, C.c_size_t, C.c_void_p, C.c_size_t,
                                       C.c_void_p, C.c_size_t, C.c_int, _u64, C.c_size_t, C.POINTER(C.c_size_t),
                                       _u64, _u64]),
    "zkml_build_verify_model_gkr_calldata": (C.c_int, [C.c_void_p, _u64, C.c_void_p, C.c_size_t, C.c_size_t,
                                                       C.c_void_p, C.c_size_t, C.c_void_p, C.c_size_t, C.c_int,
                                                       _u64, C.c_size_t, C.POINTER(C.c_size_t), _u64, _u64]),
    "zkml_p2p_inbox_create": (C.c_int, [C.c_void_p, C.c_size_t, C.c_int, C.c_int, C.c_void_p]),
    "zkml_p2p_open": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int]),
    "zkml_p2p_close": (C.c_int, [C.c_void_p]),
    "zkml_mesh_create": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_size_t, C.c_void_p]),
    "zkml_mesh_open": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int]),
    "zkml_mesh_close": (C.c_int, [C.c_void_p]),
    "zkml_prove_product_sharded_mesh": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t, C.c_size_t,
                                                  C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                                  C.c_void_p]),
    "zkml_restrict_cols_block_p2p": (C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t, C.c_size_t, C.c_size_t,
                                               C.c_void_p, C.c_size_t, C.c_uint32]),
    "zkml_reduce_matmul_layer_gkr_p2p": (C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t, _u32, C.c_void_p,
                                                   C.c_size_t, C.c_size_t, C.c_size_t, C.c_uint32,
                                                   C.POINTER(_Channel), _u32, _u32, _u32, _u32]),
    "zkml_weight_commitment": (C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t, C.c_size_t, _u64]),
    "zkml_prove_aggregated_binding": (C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t, C.POINTER(_Channel),
                                                C.c_size_t, _u64, C.c_size_t, C.POINTER(C.c_size_t)]),
    "zkml_restrict_cols_noalloc": (C.c_int, [C.c_void_p, C.c_size_t, C.c_size_t, C.c_void_p, C.c_size_t,
                                             C.c_void_p, C.c_size_t, C.c_void_p]),
    "zkml_sumcheck_load_m31": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t]),
    "zkml_sumcheck_load_qm31": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t]),
    "zkml_sumcheck_length": (C.c_size_t, [C.c_void_p]),
    "zkml_sumcheck_round": (C.c_int, [C.c_void_p, C.c_void_p, _u32]),
    "zkml_sumcheck_export": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p]),
    "zkml_sumcheck_finalize": (C.c_int, [C.c_void_p, _u32, _u32, _u32]),
    "zkml_selftest_wait_timeout": (C.c_int, [C.c_void_p, _u32]),
    "zkml_matmul_m31": (C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t, C.c_size_t, C.c_void_p, C.c_size_t,
                                  C.c_void_p]),
    "zkml_shm_exchange_open": (C.c_int, [C.c_char_p, C.c_int, C.c_int, C.c_size_t, C.c_uint64, C.c_void_p]),
    "zkml_shm_exchange_close": (C.c_int, [C.c_void_p]),
    "zkml_prove_product_sharded": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t, C.c_size_t, C.c_void_p,
                                             C.c_void_p, _u32, _u32, _u32, _u32, C.POINTER(C.c_size_t)]),
    "zkml_prove_gkr_matmul": (C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t, C.c_size_t, C.c_void_p, C.c_size_t,
                                        C.c_void_p, C.c_size_t, _u64, C.c_size_t, C.POINTER(C.c_size_t), _u64,
                                        _u64]),
}


def library_path() -> Path:
    return Path(os.environ.get("ZKML_B200_LIB", LIB_PATH))


def lib():
    """Load the CUDA library (raises if it has not been built)."""
    global _lib
    with _lib_lock:
        if _lib is None:
            path = library_path()
            if not path.exists():
                raise ImportError(f"{path} is missing: build it with `make -C stwo-ml_b200` "
                                  "(or __graft_entry__.build()); there is no CPU fallback")
            L = C.CDLL(str(path))
            for name, (res, args) in _SIGS.items():
                fn = getattr(L, name)
                fn.restype = res
                fn.argtypes = args
            _lib = L
    return _lib


def exported_symbols() -> List[str]:
    return list(_SIGS)


def _check(rc: int) -> None:
    if rc != ZKML_OK:
        msg = (lib().zkml_last_error() or b"").decode(errors="replace")
        if rc == 1:
            raise InvalidArgument(rc, msg)
        raise ZkmlError(rc, msg)


# ---------------------------------------------------------------------------
# felt252 helpers
# ---------------------------------------------------------------------------

def felt_to_limbs(x: int) -> np.ndarray:
    x %= STARK_P
    return np.array([(x >> (64 * i)) & (2**64 - 1) for i in range(4)], dtype=np.uint64)


def limbs_to_felt(a) -> int:
    return sum(int(a[i]) << (64 * i) for i in range(4))


def qm31(a: int, b: int = 0, c: int = 0, d: int = 0) -> np.ndarray:
    return np.array([a, b, c, d], dtype=np.uint32)


def as_qm31_array(x) -> np.ndarray:
    arr = np.ascontiguousarray(np.asarray(x, dtype=np.uint32))
    if arr.size == 0:
        return np.zeros((0, 4), np.uint32)
    return arr.reshape(-1, 4)


def poseidon_hash(a: int, b: int) -> int:
    out = np.zeros(4, np.uint64)
    lib().zkml_poseidon_hash(felt_to_limbs(a), felt_to_limbs(b), out)
    return limbs_to_felt(out)


def poseidon_hash_many(xs: Sequence[int]) -> int:
    arr = np.concatenate([felt_to_limbs(x) for x in xs]) if len(xs) else np.zeros(4, np.uint64)
    out = np.zeros(4, np.uint64)
    lib().zkml_poseidon_hash_many(arr, len(xs), out)
    return limbs_to_felt(out)


def hades_permutation(state: Sequence[int]) -> List[int]:
    st = np.concatenate([felt_to_limbs(x) for x in state])
    lib().zkml_hades_permutation(st)
    return [limbs_to_felt(st[4 * i:4 * i + 4]) for i in range(3)]


def securefield_to_felt(v) -> int:
    out = np.zeros(4, np.uint64)
    lib().zkml_securefield_to_felt(np.ascontiguousarray(v, np.uint32).reshape(4), out)
    return limbs_to_felt(out)


# ---------------------------------------------------------------------------
# PoseidonChannel
# ---------------------------------------------------------------------------

class PoseidonChannel:
    """Host Fiat-Shamir channel (transcript-compatible with the engine's)."""

    def __init__(self):
        self._st = _Channel()
        lib().zkml_channel_init(C.byref(self._st))

    def clone(self) -> "PoseidonChannel":
        c = PoseidonChannel.__new__(PoseidonChannel)
        c._st = _Channel.from_buffer_copy(self._st)
        return c

    @property
    def state(self) -> _Channel:
        return self._st

    def digest(self) -> int:
        return limbs_to_felt(self._st.digest)

    def n_draws(self) -> int:
        return int(self._st.n_draws)

    def hash_count(self) -> int:
        return int(self._st.hash_count)

    def mix_u64(self, v: int) -> None:
        lib().zkml_channel_mix_u64(C.byref(self._st), v)

    def mix_felt(self, v: int) -> None:
        lib().zkml_channel_mix_felt(C.byref(self._st), felt_to_limbs(v))

    def mix_secure_field(self, v) -> None:
        lib().zkml_channel_mix_qm31(C.byref(self._st), np.ascontiguousarray(v, np.uint32).reshape(4))

    def draw_felt252(self) -> int:
        out = np.zeros(4, np.uint64)
        lib().zkml_channel_draw_felt252(C.byref(self._st), out)
        return limbs_to_felt(out)

    def draw_qm31(self) -> np.ndarray:
        out = np.zeros(4, np.uint32)
        lib().zkml_channel_draw_qm31(C.byref(self._st), out)
        return out

    def draw_qm31s(self, n: int) -> np.ndarray:
        return np.stack([self.draw_qm31() for _ in range(n)]) if n else np.zeros((0, 4), np.uint32)

    def mix_poly_coeffs(self, c0, c1, c2) -> None:
        lib().zkml_channel_mix_poly_coeffs(C.byref(self._st), np.concatenate([c0, c1, c2]).astype(np.uint32))

    def mix_poly_coeffs_deg3(self, c0, c1, c2, c3) -> None:
        lib().zkml_channel_mix_poly_coeffs_deg3(C.byref(self._st),
                                                np.concatenate([c0, c1, c2, c3]).astype(np.uint32))

    def mix_felts(self, felts) -> None:
        arr = as_qm31_array(felts)
        lib().zkml_channel_mix_felts(C.byref(self._st), arr.reshape(-1) if arr.size else np.zeros(4, np.uint32),
                                     len(arr))


# ---------------------------------------------------------------------------
# Data types
# ---------------------------------------------------------------------------

@dataclass
class M31Matrix:
    """Row-major, unpadded M31 matrix (components/matmul.rs:85-116)."""
    rows: int
    cols: int
    data: object  # numpy uint32 (rows*cols) or a CUDA tensor of int32/uint32

    @staticmethod
    def from_numpy(a: np.ndarray) -> "M31Matrix":
        a = np.ascontiguousarray(a, dtype=np.uint32)
        return M31Matrix(a.shape[0], a.shape[1], a.reshape(-1))


@dataclass
class RoundPoly:
    c0: np.ndarray
    c1: np.ndarray
    c2: np.ndarray


class RoundPolys(_abc.Sequence):
    """The round polynomials of a reduction as a sequence of RoundPoly, built on access from the
    (rounds x 12) coefficient array the library wrote (views, no copies)."""

    def __init__(self, coeffs: np.ndarray):
        self.coeffs = coeffs

    def __len__(self) -> int:
        return len(self.coeffs)

    def __getitem__(self, i):
        if isinstance(i, slice):
            return [self[j] for j in range(*i.indices(len(self)))]
        row = self.coeffs[i]
        return RoundPoly(row[0:4], row[4:8], row[8:12])


@dataclass
class MatMulReduction:
    round_polys: List[RoundPoly]
    challenges: np.ndarray
    final_a_eval: np.ndarray
    final_b_eval: np.ndarray


@dataclass
class GKRClaim:
    point: np.ndarray
    value: np.ndarray


def _next_pow2(x: int) -> int:
    return 1 << max(0, (x - 1).bit_length())


def _log2(x: int) -> int:
    return x.bit_length() - 1


# ---------------------------------------------------------------------------
# Device context (GpuSumcheckExecutor::cached equivalent)
# ---------------------------------------------------------------------------

class Context:
    def __init__(self, device: int = 0):
        h = C.c_void_p()
        _check(lib().zkml_ctx_create(device, C.byref(h)))
        self.handle = h
        self.device = device

    def close(self) -> None:
        if self.handle:
            lib().zkml_ctx_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def kernel_launches(self) -> int:
        return int(lib().zkml_ctx_kernel_launches(self.handle))

    def h2d_bytes(self) -> int:
        """Host -> device bytes of this context's input-matrix uploads so far."""
        return int(lib().zkml_ctx_h2d_bytes(self.handle))

    KERNEL_CLASSES = ("restrict_cols", "restrict_rows", "sumcheck_round", "merkle", "host_sync", "host_channel")

    def enable_timing(self, enable: bool = True, classes: Optional[Sequence[str]] = None) -> None:
        """Time every kernel class (default) or only `classes`; enable=False turns timing off."""
        if not enable:
            mask = 0
        elif classes is None:
            mask = -1
        else:
            mask = 0
            for c in classes:
                mask |= 1 << self.KERNEL_CLASSES.index(c)
        _check(lib().zkml_ctx_enable_timing(self.handle, mask))

    def kernel_time(self, kernel: str) -> Tuple[float, int]:
        ms = C.c_double(0)
        n = C.c_uint64(0)
        _check(lib().zkml_ctx_kernel_time(self.handle, kernel.encode(), C.byref(ms), C.byref(n)))
        return ms.value, n.value

    def set_stream(self, stream_ptr: Optional[int]) -> None:
        _check(lib().zkml_ctx_set_stream(self.handle, C.c_void_p(stream_ptr or 0)))


_contexts = {}


def context(device: int = 0) -> Context:
    if device not in _contexts:
        _contexts[device] = Context(device)
    return _contexts[device]


class _Buf:
    """Pointer + keep-alive for a host numpy array or a device tensor."""

    def __init__(self, x, dtype=np.uint32):
        self.keep = None
        if hasattr(x, "data_ptr") and hasattr(x, "is_cuda"):
            if x.is_cuda:
                if not x.is_contiguous():
                    raise InvalidArgument(1, "device tensor must be contiguous")
                self.keep = x
                self.ptr = C.c_void_p(x.data_ptr())
                self.nbytes = x.numel() * x.element_size()
                return
            x = x.numpy()
            if x.dtype in (np.int32, np.uint32) and x.flags.c_contiguous:
                x = x.view(np.uint32)  # no copy: keeps pinned host memory pinned
        arr = np.ascontiguousarray(x, dtype=dtype)
        self.keep = arr
        self.ptr = C.c_void_p(arr.ctypes.data) if arr.size else C.c_void_p(0)
        self.nbytes = arr.nbytes


def _qm31_ptr(x) -> Tuple[C.c_void_p, np.ndarray]:
    arr = as_qm31_array(x)
    if arr.size == 0:
        arr = np.zeros((1, 4), np.uint32)
        return C.c_void_p(0), arr
    return C.c_void_p(arr.ctypes.data), arr


class GpuBackend:
    """``ZkmlOps`` on the B200 (engine/src/backend.rs:85-107)."""

    def __init__(self, device: int = 0):
        self.ctx = context(device)

    def reduce_matmul_layer(self, a: M31Matrix, b: M31Matrix, r_i, r_j, pk: int,
                            channel: PoseidonChannel) -> MatMulReduction:
        log_k = _log2(pk) if pk > 0 else 0
        r_i_p, r_i_k = _qm31_ptr(r_i)
        r_j_p, r_j_k = _qm31_ptr(r_j)
        n_ri = len(as_qm31_array(r_i))
        n_rj = len(as_qm31_array(r_j))
        abuf, bbuf = _Buf(a.data), _Buf(b.data)
        rp = np.zeros((max(log_k, 1), 12), np.uint32)
        ch = np.zeros((max(log_k, 1), 4), np.uint32)
        fa = np.zeros(4, np.uint32)
        fb = np.zeros(4, np.uint32)
        _check(lib().zkml_reduce_matmul_layer(self.ctx.handle, abuf.ptr, a.rows, a.cols, bbuf.ptr, b.rows, b.cols,
                                              r_i_p, n_ri, r_j_p, n_rj, pk, C.byref(channel.state),
                                              rp.reshape(-1), ch.reshape(-1), fa, fb))
        polys = [RoundPoly(rp[r, 0:4].copy(), rp[r, 4:8].copy(), rp[r, 8:12].copy()) for r in range(log_k)]
        return MatMulReduction(polys, ch[:log_k].copy(), fa, fb)

    def evaluate_mle_at_point(self, mle, point) -> np.ndarray:
        buf = _Buf(mle)
        p_ptr, p_keep = _qm31_ptr(point)
        n_vars = len(as_qm31_array(point))
        out = np.zeros(4, np.uint32)
        _check(lib().zkml_evaluate_mle(self.ctx.handle, buf.ptr, n_vars, p_ptr, out))
        return out

    def restrict_mle(self, mle, assignments) -> np.ndarray:
        buf = _Buf(mle)
        n_evals = buf.nbytes // 16
        p_ptr, p_keep = _qm31_ptr(assignments)
        n_assign = len(as_qm31_array(assignments))
        out = np.zeros((max(n_evals >> n_assign, 1), 4), np.uint32)
        _check(lib().zkml_restrict_mle(self.ctx.handle, buf.ptr, n_evals, p_ptr, n_assign, out.reshape(-1)))
        return out[:n_evals >> n_assign]


_fast_fns = {}


def _fast_fn(name: str, nargs: int):
    """The C entry point `name` with every argument passed as a plain integer (pointer or
    size): no per-call ctypes array validation on the hot path."""
    f = _fast_fns.get(name)
    if f is None:
        addr = C.cast(getattr(lib(), name), C.c_void_p).value
        f = C.CFUNCTYPE(C.c_int, *([C.c_void_p] * nargs))(addr)
        _fast_fns[name] = f
    return f


def reduce_matmul_layer_with_backend(output_claim: GKRClaim, a: M31Matrix, b: M31Matrix, m: int, k: int, n: int,
                                     channel: PoseidonChannel, backend: Optional[GpuBackend] = None
                                     ) -> Tuple[MatMulReduction, GKRClaim]:
    """gkr/prover.rs:5959-6073 -- transcript wrapper around ``reduce_matmul_layer``."""
    backend = backend or GpuBackend()
    pm, pk, pn = _next_pow2(a.rows), _next_pow2(a.cols), _next_pow2(b.cols)
    log_m, log_k, log_n = _log2(pm), _log2(pk), _log2(pn)
    point = as_qm31_array(output_claim.point)
    abuf, bbuf = _Buf(a.data), _Buf(b.data)
    if (a.rows, a.cols, b.cols) != (m, k, n) or b.rows != k:
        raise InvalidArgument(1, "matrix shapes do not match (m, k, n)")
    # one allocation (and one pointer lookup) for the point, the claimed value and every output:
    # round polynomials, final a / b, next point
    npw = point.size
    n_rp = 12 * max(log_k, 1)
    buf = np.empty(npw + 4 + n_rp + 8 + 4 * max(log_m + log_k, 1), np.uint32)
    buf[:npw] = point.reshape(-1)
    buf[npw:npw + 4] = np.asarray(output_claim.value, np.uint32).reshape(4)
    base = buf.ctypes.data
    o_rp = npw + 4
    o_fa = o_rp + n_rp
    o_nx = o_fa + 8
    _check(_fast_fn("zkml_reduce_matmul_layer_gkr", 14)(
        backend.ctx.handle.value, base if npw else None, len(point), base + 4 * npw, abuf.ptr.value, m, k,
        bbuf.ptr.value, n, C.addressof(channel.state), base + 4 * o_rp, base + 4 * o_fa, base + 4 * o_fa + 16,
        base + 4 * o_nx))
    fa = buf[o_fa:o_fa + 4]
    fb = buf[o_fa + 4:o_fa + 8]
    nxt = buf[o_nx:].reshape(-1, 4)
    # views of this call's own fresh array (no per-round copies)
    red = MatMulReduction(RoundPolys(buf[o_rp:o_rp + n_rp].reshape(-1, 12)[:log_k]), nxt[log_m:log_m + log_k],
                          fa, fb)
    return red, GKRClaim(nxt[:log_m + log_k], fa.copy())


# ---------------------------------------------------------------------------
# Merkle commitment, MLE opening, single-layer GKR proof
# ---------------------------------------------------------------------------

DEFAULT_MLE_N_QUERIES = 10  # STWO_MLE_N_QUERIES default (crypto/mle_opening.rs:42-58)


def mle_n_queries() -> int:
    """STWO_MLE_N_QUERIES (2..=20, default 10), as the reference reads it."""
    try:
        v = int(os.environ.get("STWO_MLE_N_QUERIES", ""))
        if 2 <= v <= 20:
            return v
    except ValueError:
        pass
    return DEFAULT_MLE_N_QUERIES


def _felts(buf: np.ndarray, n: int) -> List[int]:
    return [limbs_to_felt(buf[4 * i:4 * i + 4]) for i in range(n)]


def matmul_m31(a, b, out=None, device: int = 0):
    """C = A * B mod p (forward pass, gpu_matmul_m31_full).  a: (m, k), b: (k, n) M31 as numpy
    arrays or CUDA tensors; returns a numpy (m, n) uint32 array, or writes `out` (a CUDA int32
    tensor of m * n elements) in place."""
    am, bm = as_matrix(a), as_matrix(b)
    if am.cols != bm.rows:
        raise InvalidArgument(1, "A.cols must equal B.rows")
    ab, bb = _Buf(am.data), _Buf(bm.data)
    if out is None:
        res = np.zeros((am.rows, bm.cols), np.uint32)
        _check(lib().zkml_matmul_m31(context(device).handle, ab.ptr, am.rows, am.cols, bb.ptr, bm.cols,
                                     res.ctypes.data_as(C.c_void_p)))
        return res
    ob = _Buf(out)
    _check(lib().zkml_matmul_m31(context(device).handle, ab.ptr, am.rows, am.cols, bb.ptr, bm.cols, ob.ptr))
    return out


def as_matrix(x) -> "M31Matrix":
    if isinstance(x, M31Matrix):
        return x
    if hasattr(x, "is_cuda"):
        return M31Matrix(int(x.shape[0]), int(x.shape[1]), x.reshape(-1))
    return M31Matrix.from_numpy(np.asarray(x))


def commit_mle_root(evals, device: int = 0) -> int:
    """commit_mle_root_only: Poseidon Merkle root of QM31 evaluations."""
    buf = _Buf(evals)
    out = np.zeros(4, np.uint64)
    _check(lib().zkml_commit_mle_root(context(device).handle, buf.ptr, buf.nbytes // 16, out))
    return limbs_to_felt(out)


@dataclass
class MleOpening:
    commitment: int
    calldata: List[int]  # serialize_mle_opening_proof layout


def prove_mle_opening(evals, point, channel: PoseidonChannel, n_queries: Optional[int] = None,
                      device: int = 0) -> MleOpening:
    """prove_mle_opening_with_commitment (crypto/mle_opening.rs:1654-1916)."""
    buf = _Buf(evals)
    n_evals = buf.nbytes // 16
    n_vars = n_evals.bit_length() - 1
    if n_evals != 1 << n_vars:
        raise InvalidArgument(1, "MLE length must be a power of two")
    p_ptr, p_keep = _qm31_ptr(point)
    nq = mle_n_queries() if n_queries is None else n_queries
    cap = 64 + (nq + 1) * (2 + n_vars * (10 + 2 * (n_vars + 1)))
    out = np.empty(4 * cap, np.uint64)  # the library writes every reported felt
    com = np.zeros(4, np.uint64)
    ln = C.c_size_t(0)
    _check(lib().zkml_prove_mle_opening(context(device).handle, buf.ptr, n_vars, p_ptr, C.byref(channel.state), nq,
                                        com, out, cap, C.byref(ln)))
    return MleOpening(limbs_to_felt(com), _felts(out, ln.value))


def io_commitment(inp: np.ndarray, out: np.ndarray) -> int:
    inp = np.ascontiguousarray(inp, np.uint32)
    out = np.ascontiguousarray(out, np.uint32)
    res = np.zeros(4, np.uint64)
    _check(lib().zkml_io_commitment(inp.reshape(-1), inp.shape[0], inp.shape[1], out.reshape(-1), out.shape[0],
                                    out.shape[1], res))
    return limbs_to_felt(res)


@dataclass
class GKRMatMulProof:
    calldata: List[int]  # serialize_gkr_model_proof
    final_digest: int
    io_commitment: int
    raw: np.ndarray       # calldata as 4 x u64 limbs per felt


def prove_gkr_matmul(inp: M31Matrix, weight: M31Matrix, policy_commitment: Optional[int] = None,
                     n_queries: Optional[int] = None, device: int = 0) -> GKRMatMulProof:
    """prove_gkr for GraphBuilder::new((m, k)).linear(n), Sequential weight binding."""
    ibuf, wbuf = _Buf(inp.data), _Buf(weight.data)
    m, k, n = inp.rows, inp.cols, weight.cols
    if weight.rows != k:
        raise InvalidArgument(1, "weight rows must equal input cols")
    nq = mle_n_queries() if n_queries is None else n_queries
    nv = _log2(_next_pow2(n)) + _log2(_next_pow2(k))
    cap = 256 + 24 * (_log2(_next_pow2(k)) + _log2(_next_pow2(m))) + (nq + 1) * (2 + nv * (10 + 2 * (nv + 1)))
    buf = np.zeros(4 * cap, np.uint64)
    ln = C.c_size_t(0)
    dig = np.zeros(4, np.uint64)
    io = np.zeros(4, np.uint64)
    pol = None
    if policy_commitment:
        pol = felt_to_limbs(policy_commitment)
    _check(lib().zkml_prove_gkr_matmul(context(device).handle, ibuf.ptr, m, k, wbuf.ptr, n,
                                       C.c_void_p(pol.ctypes.data) if pol is not None else None, nq, buf, cap,
                                       C.byref(ln), dig, io))
    return GKRMatMulProof(_felts(buf, ln.value), limbs_to_felt(dig), limbs_to_felt(io), buf[:4 * ln.value].copy())


# ---------------------------------------------------------------------------
# LogUp activation layer
# ---------------------------------------------------------------------------

class ActivationType:
    """components/activation.rs:39-71 type tags."""
    ReLU = 1
    GELU = 2
    Sigmoid = 3
    Softmax = 4
    SiLU = 5

    @staticmethod
    def table_log_size(tag: int) -> int:
        return 20 if tag == ActivationType.Softmax else 16


def activation_table(tag: int) -> np.ndarray:
    """The activation lookup table (host)."""
    n = 1 << ActivationType.table_log_size(tag)
    out = np.zeros(n, np.uint32)
    ln = C.c_size_t(0)
    _check(lib().zkml_activation_table(tag, out, n, C.byref(ln)))
    return out


@dataclass
class ActivationLogUpProof:
    """LayerProof::Activation record (serialize_gkr_model_proof).  `raw` holds the calldata as
    4 x u64 limbs per felt; `calldata` converts it to Python integers on first use (the record
    carries the 2^16 table multiplicities, so the conversion costs far more than the proof)."""
    raw: np.ndarray
    input_eval: np.ndarray  # next claim value

    @property
    def calldata(self) -> List[int]:
        if not hasattr(self, "_calldata"):
            self._calldata = _felts(self.raw, self.raw.size // 4)
        return self._calldata


def reduce_activation_layer(output_claim: GKRClaim, inp: M31Matrix, activation_type: int,
                            channel: PoseidonChannel, device: int = 0) -> Tuple[ActivationLogUpProof, GKRClaim]:
    """gkr/prover.rs:6390-6600 (LogUp path)."""
    buf = _Buf(inp.data)
    pt_ptr, pt_keep = _qm31_ptr(output_claim.point)
    n_point = len(as_qm31_array(output_claim.point))
    tsize = 1 << ActivationType.table_log_size(activation_type)
    cap = tsize + 64 + 16 * (n_point + 40)
    out = np.empty(4 * cap, np.uint64)  # the library writes every reported felt
    ln = C.c_size_t(0)
    ie = np.zeros(4, np.uint32)
    _check(lib().zkml_reduce_activation_logup(context(device).handle, buf.ptr, inp.rows, inp.cols, activation_type,
                                              pt_ptr, n_point, np.ascontiguousarray(output_claim.value, np.uint32),
                                              C.byref(channel.state), out, cap, C.byref(ln), ie))
    proof = ActivationLogUpProof(out[:4 * ln.value], ie)
    return proof, GKRClaim(as_qm31_array(output_claim.point).copy(), ie.copy())


def piecewise_activation_enabled() -> bool:
    """STWO_PIECEWISE_ACTIVATION (default on; 0/false/no/off select the LogUp path),
    components/activation.rs:365-373."""
    v = os.environ.get("STWO_PIECEWISE_ACTIVATION")
    if v is None:
        return True
    return v.strip().lower() not in ("0", "false", "no", "off")


def reduce_activation_layer_piecewise(output_claim: GKRClaim, inp: M31Matrix, activation_type: int,
                                      channel: PoseidonChannel, device: int = 0
                                      ) -> Tuple[ActivationLogUpProof, GKRClaim]:
    """gkr/prover.rs:7006-7228.  Returns the LayerProof::Activation record (piecewise proof)
    and the next claim (the sumcheck challenges, the input evaluation)."""
    buf = _Buf(inp.data)
    pt_ptr, pt_keep = _qm31_ptr(output_claim.point)
    n_point = len(as_qm31_array(output_claim.point))
    cap = 64 + 12 * n_point + 4 * 24
    out = np.empty(4 * cap, np.uint64)  # the library writes every reported felt
    ln = C.c_size_t(0)
    ie = np.zeros(4, np.uint32)
    nxt = np.zeros((max(n_point, 1), 4), np.uint32)
    _check(lib().zkml_reduce_activation_piecewise(context(device).handle, buf.ptr, inp.rows, inp.cols,
                                                  activation_type, pt_ptr, n_point,
                                                  np.ascontiguousarray(output_claim.value, np.uint32),
                                                  C.byref(channel.state), out, cap, C.byref(ln), ie,
                                                  nxt.reshape(-1)))
    proof = ActivationLogUpProof(out[:4 * ln.value], ie)
    return proof, GKRClaim(nxt[:n_point].copy(), ie.copy())


def reduce_activation_layer_relu(output_claim: GKRClaim, inp: M31Matrix, channel: PoseidonChannel,
                                 device: int = 0) -> Tuple[ActivationLogUpProof, GKRClaim]:
    """gkr/prover.rs:6700-6890 (ReLU, algebraic).  Returns the LayerProof::Activation record and
    the next claim (the sumcheck challenges, the input evaluation)."""
    buf = _Buf(inp.data)
    pt_ptr, pt_keep = _qm31_ptr(output_claim.point)
    n_point = len(as_qm31_array(output_claim.point))
    cap = 256 + 12 * n_point
    out = np.empty(4 * cap, np.uint64)  # the library writes every reported felt
    ln = C.c_size_t(0)
    ie = np.zeros(4, np.uint32)
    nxt = np.zeros((max(n_point, 1), 4), np.uint32)
    _check(lib().zkml_reduce_activation_relu(context(device).handle, buf.ptr, inp.rows, inp.cols, pt_ptr, n_point,
                                             np.ascontiguousarray(output_claim.value, np.uint32),
                                             C.byref(channel.state), out, cap, C.byref(ln), ie, nxt.reshape(-1)))
    return ActivationLogUpProof(out[:4 * ln.value], ie), GKRClaim(nxt[:n_point].copy(), ie.copy())


class _ChainLayer(C.Structure):
    _fields_ = [("type", C.c_int), ("weight", C.c_void_p), ("n", C.c_size_t), ("src", C.c_longlong),
                ("lhs", C.c_longlong)]


CHAIN_PREV = -2
_CHAIN_KINDS = {"linear": 0, "relu": 1, "rmsnorm": 2, "add": 3, "mul": 4, "layernorm": 5, "activation": 6}
# ActivationType::type_tag (components/activation.rs:50-60) of the non-ReLU activations
ACTIVATION_TAGS = {"gelu": 2, "sigmoid": 3, "softmax": 4, "silu": 5}
CHAIN_ACTIVATION_LOGUP = 4
CHAIN_MESH = 8


def piecewise_activation_enabled() -> bool:
    """STWO_PIECEWISE_ACTIVATION as the reference reads it (components/activation.rs:365-373):
    on unless set to 0 / false / no / off."""
    v = os.environ.get("STWO_PIECEWISE_ACTIVATION")
    if v is None:
        return True
    return v.strip().lower() not in ("0", "false", "no", "off")


@dataclass
class GKRChainProof:
    raw: np.ndarray       # serialize_gkr_model_proof (or verify_model_gkr calldata), 4 x u64 limbs per felt
    final_digest: int
    io_commitment: int

    @property
    def calldata(self) -> List[int]:
        return _felts(self.raw, self.raw.size // 4)


def _chain_args(inp, layers, n_queries):
    """ctypes layer array, buffers to keep alive and a calldata capacity for `layers`, each
    (kind, arg[, src]): ("linear", weight (in_width, n)), ("relu", None), ("activation", type: "silu" /
    "gelu" / "sigmoid" / "softmax" or its tag), ("rmsnorm", None), ("layernorm", None), ("add", lhs_layer),
    ("mul", lhs_layer); src = the layer feeding this one (None: the previous layer, -1: the model
    input).  The Add / Mul rhs operand is src's output."""
    im = as_matrix(inp)
    ib = _Buf(im.data)
    keep = [ib]
    arr = (_ChainLayer * len(layers))()
    widths = [im.cols]  # widths[l + 1]: layer l's output width; widths[0]: the input's
    nv_max, n_lin, n_bin, n_act_mult = 0, 0, 0, 0
    for i, spec in enumerate(layers):
        kind, arg = spec[0], spec[1]
        src = spec[2] if len(spec) > 2 and spec[2] is not None else CHAIN_PREV
        if kind not in _CHAIN_KINDS:
            raise InvalidArgument(1, f"layer {i}: unknown kind {kind}")
        s_eff = i - 1 if src == CHAIN_PREV else src
        if not -1 <= s_eff < i:
            raise InvalidArgument(1, f"layer {i}: input layer {src} is not a lower layer")
        width = widths[s_eff + 1]
        arr[i].type, arr[i].weight, arr[i].n, arr[i].src, arr[i].lhs = _CHAIN_KINDS[kind], None, 0, src, -1
        if kind == "linear":
            wm = as_matrix(arg)
            if wm.rows != width:
                raise InvalidArgument(1, f"layer {i}: weight rows {wm.rows} != input width {width}")
            wb = _Buf(wm.data)
            keep.append(wb)
            arr[i].weight, arr[i].n = wb.ptr.value, wm.cols
            nv_max = max(nv_max, _log2(_next_pow2(wm.rows)) + _log2(_next_pow2(wm.cols)))
            width = wm.cols
            n_lin += 1
        elif kind in ("add", "mul"):
            arr[i].lhs = int(arg)
            n_bin += 1
        elif kind == "activation":
            tag = ACTIVATION_TAGS[arg.lower()] if isinstance(arg, str) else int(arg)
            if tag not in ACTIVATION_TAGS.values():
                raise InvalidArgument(1, f"layer {i}: activation must be GELU, Sigmoid, Softmax or SiLU")
            arr[i].n = tag
            n_act_mult += 1 << (20 if tag == 4 else 16)
        widths.append(width)
    nq = mle_n_queries() if n_queries is None else n_queries
    nv_all = _log2(_next_pow2(im.rows)) + max(nv_max, max(_log2(_next_pow2(w)) for w in widths) + 1)
    n_norm = sum(1 for spec in layers if spec[0] in ("rmsnorm", "layernorm"))
    per_open = 64 + (nq + 1) * (2 + nv_max * (10 + 2 * (nv_max + 1)))
    cap = 256 + len(layers) * (200 + 12 * nv_all) + (n_lin + n_bin) * per_open + n_bin * (60 + 16 * nv_all)
    cap += n_norm * ((1 << 16) + 2 * _next_pow2(im.rows) + 200 + 60 * (nv_all + 2))
    cap += 2 * im.rows * max(widths) + n_act_mult
    return im, ib, arr, keep, nq, cap


def prove_gkr_chain(inp, layers, policy_commitment: Optional[int] = None, n_queries: Optional[int] = None,
                    legacy_activation_record: bool = False, v1_layout: bool = False,
                    device: int = 0, activation_logup: Optional[bool] = None, mesh=None) -> GKRChainProof:
    """prove_gkr (gkr/prover.rs:1500-2251) for GraphBuilder::new(inp.shape) followed by `layers`
    (see _chain_args; Add / Mul layers defer their skip branch), Sequential weight binding.
    raw: serialize_gkr_model_proof, or with v1_layout the verify_model_gkr calldata from
    proof_data on (deferred proofs and their openings included).  Activation layers take the
    LogUp reduction when activation_logup is true, the piecewise one when false; None follows
    STWO_PIECEWISE_ACTIVATION as the reference does (prover.rs:1765-1790).  With a
    distributed.PeerMesh, every rank of the mesh makes this call and the weight openings'
    Merkle hashing is split across them (same proof on every rank)."""
    if activation_logup is None:
        activation_logup = not piecewise_activation_enabled()
    im, ib, arr, keep, nq, cap = _chain_args(inp, layers, n_queries)
    out = np.empty(4 * cap, np.uint64)  # the library writes every reported felt
    ln = C.c_size_t(0)
    dig = np.zeros(4, np.uint64)
    io = np.zeros(4, np.uint64)
    pol = felt_to_limbs(policy_commitment) if policy_commitment else None
    flags = (1 if legacy_activation_record else 0) | (2 if v1_layout else 0)
    flags |= CHAIN_ACTIVATION_LOGUP if activation_logup else 0
    if mesh is not None:
        flags |= CHAIN_MESH
        device = mesh.ctx.device
    _check(lib().zkml_prove_gkr_chain(context(device).handle, ib.ptr, im.rows, im.cols, C.cast(arr, C.c_void_p),
                                      len(layers), C.c_void_p(pol.ctypes.data) if pol is not None else None, nq,
                                      flags, out, cap, C.byref(ln), dig, io))
    return GKRChainProof(out[:4 * ln.value], limbs_to_felt(dig), limbs_to_felt(io))


_DESCRIPTOR_TAGS = {"linear": 0, "add": 1, "mul": 2, "relu": 3, "activation": 3, "layernorm": 4, "rmsnorm": 8}


def circuit_descriptor(layers) -> List[int]:
    """build_circuit_descriptor (starknet.rs:1591-1617): [layer count, tag of each layer from
    the output to the input] with MatMul 0, Add 1, Mul 2, Activation 3, LayerNorm 4, RMSNorm 8."""
    return [len(layers)] + [_DESCRIPTOR_TAGS[spec[0]] for spec in reversed(layers)]


def build_register_gkr_calldata(model_id: int, weight_commitments: Sequence[int], layers) -> List[str]:
    """build_register_gkr_calldata (starknet.rs:1619-1640): the sncast calldata of
    register_model_gkr(model_id, weight_commitments, circuit_descriptor)."""
    desc = circuit_descriptor(layers)
    return ([f"0x{model_id:x}", str(len(weight_commitments))] + [f"0x{c:x}" for c in weight_commitments]
            + [str(len(desc))] + [str(t) for t in desc])


def verify_calldata_weight_commitments(calldata: Sequence[int], layers) -> List[int]:
    """The walk's weight commitments (GKRProof::weight_commitments, without the deferred
    branches') of a verify_model_gkr calldata that build_verify_model_gkr_calldata built for
    `layers`: one per Linear layer the walk reaches (a Mul layer takes its lower input out of
    the walk, prover.rs:1740-1750)."""
    skipped = set()
    for i, spec in enumerate(layers):
        if spec[0] == "mul":
            src = i - 1 if len(spec) < 3 or spec[2] is None or spec[2] == CHAIN_PREV else spec[2]
            skipped.add(min(int(spec[1]), src))
    n_walk = sum(1 for i, spec in enumerate(layers) if spec[0] == "linear" and i not in skipped)
    i = 2 + calldata[1] + 2
    i += 1 + calldata[i]  # matmul dims
    i += 1 + calldata[i]  # dequantize bits
    i += 1 + calldata[i]  # proof_data
    return list(calldata[i + 1:i + 1 + n_walk])


def build_verify_model_gkr_calldata(model_id: int, inp, layers, policy_commitment: Optional[int] = None,
                                    n_queries: Optional[int] = None, device: int = 0,
                                    activation_logup: Optional[bool] = None) -> GKRChainProof:
    """build_verify_model_gkr_calldata (starknet.rs:2837-2852): the proof of the circuit and the
    whole verify_model_gkr(model_id, raw_io_data, circuit_depth, num_layers, matmul_dims,
    dequantize_bits, proof_data, weight_commitments, weight_opening_proofs) calldata."""
    if activation_logup is None:
        activation_logup = not piecewise_activation_enabled()
    im, ib, arr, keep, nq, cap = _chain_args(inp, layers, n_queries)
    out = np.empty(4 * cap, np.uint64)
    ln = C.c_size_t(0)
    dig = np.zeros(4, np.uint64)
    io = np.zeros(4, np.uint64)
    pol = felt_to_limbs(policy_commitment) if policy_commitment else None
    _check(lib().zkml_build_verify_model_gkr_calldata(
        context(device).handle, felt_to_limbs(model_id), ib.ptr, im.rows, im.cols, C.cast(arr, C.c_void_p),
        len(layers), C.c_void_p(pol.ctypes.data) if pol is not None else None, nq,
        CHAIN_ACTIVATION_LOGUP if activation_logup else 0, out, cap, C.byref(ln), dig, io))
    return GKRChainProof(out[:4 * ln.value], limbs_to_felt(dig), limbs_to_felt(io))


@dataclass
class RMSNormProof:
    """LayerProof::RMSNorm record (serialize_gkr_model_proof).  `raw` holds the calldata as
    4 x u64 limbs per felt; `calldata` converts it to Python integers on first use."""
    raw: np.ndarray
    input_eval: np.ndarray   # next claim value
    output_eval: np.ndarray  # the RMSNorm output MLE at the claim point

    @property
    def calldata(self) -> List[int]:
        if not hasattr(self, "_calldata"):
            self._calldata = _felts(self.raw, self.raw.size // 4)
        return self._calldata


def reduce_rmsnorm_layer(output_claim: GKRClaim, inp: M31Matrix, dim: int, channel: PoseidonChannel,
                         gamma=None, device: int = 0) -> Tuple[RMSNormProof, GKRClaim]:
    """gkr/prover.rs:8424-8790 (reduce_rmsnorm_layer_with_gamma).  `gamma` is the optional
    learned per-column scale (M31 values, numpy or a CUDA tensor); STWO_SKIP_RMS_SQ_PROOF in
    the environment leaves out the RMS^2 sumcheck, as in the reference."""
    buf = _Buf(inp.data)
    gbuf = None if gamma is None else _Buf(gamma)
    pt_ptr, pt_keep = _qm31_ptr(output_claim.point)
    n_point = len(as_qm31_array(output_claim.point))
    pr = 1 << max(0, (inp.rows - 1).bit_length())
    cap = (1 << 16) + pr + 64 + 40 * (n_point + 2)
    out = np.empty(4 * cap, np.uint64)  # the library writes every reported felt
    ln = C.c_size_t(0)
    ie = np.zeros(4, np.uint32)
    _check(lib().zkml_reduce_rmsnorm(context(device).handle, buf.ptr, inp.rows, inp.cols, dim,
                                     None if gbuf is None else gbuf.ptr, 0 if gbuf is None else gbuf.nbytes // 4,
                                     pt_ptr, n_point, np.ascontiguousarray(output_claim.value, np.uint32),
                                     C.byref(channel.state), out, cap, C.byref(ln), ie))
    raw = out[:4 * ln.value]
    oe = np.array([raw[4 * (5 + i)] for i in range(4)], np.uint32)
    return RMSNormProof(raw, ie, oe), GKRClaim(as_qm31_array(output_claim.point).copy(), ie.copy())


def reduce_layernorm_layer(output_claim: GKRClaim, inp: M31Matrix, dim: int, channel: PoseidonChannel,
                           device: int = 0) -> Tuple[RMSNormProof, GKRClaim]:
    """gkr/prover.rs:7944-8354 (reduce_layernorm_layer): the LayerProof::LayerNorm record and
    the next claim (same point, the input's evaluation)."""
    buf = _Buf(inp.data)
    pt_ptr, pt_keep = _qm31_ptr(output_claim.point)
    n_point = len(as_qm31_array(output_claim.point))
    pr = 1 << max(0, (inp.rows - 1).bit_length())
    cap = (1 << 16) + 2 * pr + 200 + 60 * (n_point + 2)
    out = np.empty(4 * cap, np.uint64)  # the library writes every reported felt
    ln = C.c_size_t(0)
    ie = np.zeros(4, np.uint32)
    _check(lib().zkml_reduce_layernorm(context(device).handle, buf.ptr, inp.rows, inp.cols, dim, pt_ptr, n_point,
                                       np.ascontiguousarray(output_claim.value, np.uint32), C.byref(channel.state),
                                       out, cap, C.byref(ln), ie))
    raw = out[:4 * ln.value]
    oe = np.array([raw[4 * (5 + i)] for i in range(4)], np.uint32)
    return RMSNormProof(raw, ie, oe), GKRClaim(as_qm31_array(output_claim.point).copy(), ie.copy())


# ---------------------------------------------------------------------------
# Aggregated weight binding
# ---------------------------------------------------------------------------

class _WeightClaim(C.Structure):
    _fields_ = [("weight", C.c_void_p), ("rows", C.c_size_t), ("cols", C.c_size_t),
                ("matrix_index", C.c_size_t), ("eval_point", C.c_void_p),
                ("expected_value", C.c_uint32 * 4), ("commitment", C.c_uint64 * 4)]


def weight_commitment(weight, device: int = 0) -> int:
    """commit_mle_root_only(matrix_to_mle_col_major_padded(weight)) (gkr/prover.rs:1137-1139)."""
    wm = as_matrix(weight)
    buf = _Buf(wm.data)
    out = np.zeros(4, np.uint64)
    _check(lib().zkml_weight_commitment(context(device).handle, buf.ptr, wm.rows, wm.cols, out))
    return limbs_to_felt(out)


@dataclass
class AggregatedWeightClaim:
    """crypto/aggregated_opening.rs:99-112, carrying its weight matrix (the reference's
    WeightSource supplies it separately)."""
    weight: object            # M31Matrix, numpy (rows, cols) or a CUDA tensor
    matrix_index: int
    eval_point: object        # (n, 4) QM31, n = log2(padded rows * padded cols)
    expected_value: object    # (4,) QM31
    commitment: int           # weight_commitment(weight)


@dataclass
class AggregatedBindingProof:
    """serialize_aggregated_binding_proof layout; `raw` is 4 x u64 limbs per felt."""
    raw: np.ndarray

    @property
    def calldata(self) -> List[int]:
        return _felts(self.raw, self.raw.size // 4)


def prove_aggregated_binding(claims: List[AggregatedWeightClaim], channel: PoseidonChannel,
                             n_queries: Optional[int] = None, device: int = 0) -> AggregatedBindingProof:
    """prove_aggregated_binding_streaming (crypto/aggregated_opening.rs:1647-1719)."""
    keep = []
    arr = (_WeightClaim * len(claims))()
    n_max = 0
    for i, c in enumerate(claims):
        wm = as_matrix(c.weight)
        wb = _Buf(wm.data)
        pt = np.ascontiguousarray(as_qm31_array(c.eval_point), np.uint32)
        keep += [wb, pt]
        arr[i].weight = wb.ptr.value
        arr[i].rows, arr[i].cols = wm.rows, wm.cols
        arr[i].matrix_index = c.matrix_index
        arr[i].eval_point = pt.ctypes.data if pt.size else None
        v = np.asarray(c.expected_value, np.uint32).reshape(4)
        limbs = felt_to_limbs(c.commitment)
        for j in range(4):
            arr[i].expected_value[j] = int(v[j])
            arr[i].commitment[j] = int(limbs[j])
        n_max = max(n_max, _log2(_next_pow2(wm.rows)) + _log2(_next_pow2(wm.cols)))
    nq = mle_n_queries() if n_queries is None else n_queries
    ng = n_max + _log2(_next_pow2(len(claims)))
    cap = 64 + 12 * ng + _next_pow2(len(claims)) + (nq + 1) * (2 + ng * (10 + 2 * (ng + 1)))
    out = np.empty(4 * cap, np.uint64)  # the library writes every reported felt
    ln = C.c_size_t(0)
    _check(lib().zkml_prove_aggregated_binding(context(device).handle, C.cast(arr, C.c_void_p), len(claims),
                                               C.byref(channel.state), nq, out, cap, C.byref(ln)))
    return AggregatedBindingProof(out[:4 * ln.value])


# ---------------------------------------------------------------------------
# Allocation-free restriction (no reference counterpart)
# ---------------------------------------------------------------------------

NOALLOC_MAX_ROWS = 65536
NOALLOC_MAX_COLS = 1 << 20


def restrict_cols_noalloc(b, rows: int, cols: int, r_j, out, stream_ptr: Optional[int] = None) -> None:
    """Column restriction into a caller-provided device buffer, allocating nothing.

    For callers that cannot allocate GPU memory: ``b`` (rows x cols M31) and
    ``out`` (>= rows QM31) are CUDA tensors the caller owns; the scratch is a
    fixed array inside the library (rows <= 65536, cols <= 2^20).  Calls that
    overlap on the GPU share that array and race.
    """
    bb, ob = _Buf(b), _Buf(out)
    r_ptr, r_keep = _qm31_ptr(r_j)
    n_rj = len(as_qm31_array(r_j))
    _check(lib().zkml_restrict_cols_noalloc(bb.ptr, rows, cols, r_ptr, n_rj, ob.ptr, ob.nbytes // 16,
                                            C.c_void_p(stream_ptr or 0)))
