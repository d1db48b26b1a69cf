"""Forward M31 GEMM (zkml_matmul_m31) against the oracle's C = A * B mod p."""
import numpy as np
import pytest

import oracle_lib
from helpers import int_matrix_m31, uniform_m31

P = (1 << 31) - 1


def oracle_matmul(a, b):
    a = np.ascontiguousarray(a, np.uint32)
    b = np.ascontiguousarray(b, np.uint32)
    m, k = a.shape
    n = b.shape[1]
    c = np.zeros(m * n, np.uint32)
    oracle_lib.lib().orc_matmul_m31(a.reshape(-1), m, k, b.reshape(-1), n, c, 8)
    return c.reshape(m, n)


def test_oracle_matmul_small_reference():
    """The oracle product itself on a hand-checkable case (CPU)."""
    a = np.array([[1, 2], [P - 1, 3]], np.uint32)
    b = np.array([[4, 5, 6], [7, 8, P - 2]], np.uint32)
    want = (a.astype(object) @ b.astype(object)) % P
    np.testing.assert_array_equal(oracle_matmul(a, b), want.astype(np.uint32))


@pytest.mark.gpu
@pytest.mark.parametrize("m,k,n,kind", [(64, 5120, 1024, "int8"), (3, 36, 17, "uniform"), (65, 100, 40, "uniform"),
                                        (16, 8200, 24, "uniform"), (5, 33, 7, "uniform"), (8, 64, 9, "edge")])
def test_matmul_m31_matches_oracle(m, k, n, kind):
    import zkml_b200 as Z
    if kind == "int8":
        a, b = int_matrix_m31(m, k, 1), int_matrix_m31(k, n, 2)
    elif kind == "uniform":
        a, b = uniform_m31(m * k, 3).reshape(m, k), uniform_m31(k * n, 4).reshape(k, n)
    else:  # field edges, including the non-canonical zero P
        rng = np.random.default_rng(1)
        vals = np.array([0, 1, P - 1, P, P - 2, 1 << 30], np.uint32)
        a, b = rng.choice(vals, (m, k)), rng.choice(vals, (k, n))
    got = Z.matmul_m31(a, b)
    np.testing.assert_array_equal(got, oracle_matmul(a, b))


@pytest.mark.gpu
def test_matmul_m31_device_output_and_bad_values():
    import torch
    import zkml_b200 as Z
    a, b = uniform_m31(32 * 96, 5).reshape(32, 96), uniform_m31(96 * 48, 6).reshape(96, 48)
    ta = torch.from_numpy(a.view(np.int32)).cuda()
    tb = torch.from_numpy(b.view(np.int32)).cuda()
    out = torch.zeros(32 * 48, dtype=torch.int32, device="cuda")
    Z.matmul_m31(ta.reshape(32, 96), tb.reshape(96, 48), out=out)
    np.testing.assert_array_equal(out.cpu().numpy().view(np.uint32).reshape(32, 48), oracle_matmul(a, b))
    bad = b.copy()
    bad[3, 4] = 0x80000001
    with pytest.raises(Z.InvalidArgument):
        Z.matmul_m31(a, bad)
    np.testing.assert_array_equal(Z.matmul_m31(a, b), oracle_matmul(a, b))  # context still usable


def signed_m31(v):
    v = np.asarray(v, np.int64)
    return np.where(v >= 0, v, P + v).astype(np.uint32)


@pytest.mark.gpu
@pytest.mark.parametrize("m,k,n,arange,brange", [
    (64, 5120, 1536, 32767, 127),       # int16 activations x int8 weights: the signed-digit path
    (7, 33, 19, 32000, 127),            # k not a multiple of 4 or 32
    (64, 5120, 96, 32768, 128),         # ranges just past the digits: full-kernel fallback
    (32, 1000, 64, 40000, 127),
    (16, 300, 40, 100, 127),
])
def test_matmul_m31_narrow_values(m, k, n, arange, brange):
    import zkml_b200 as Z
    rng = np.random.default_rng(m + k + n)
    a = signed_m31(rng.integers(-arange, arange + 1, (m, k)))
    b = signed_m31(rng.integers(-brange, brange + 1, (k, n)))
    # the digit boundaries themselves
    a.flat[0], a.flat[1] = signed_m31(-32768), signed_m31(min(arange, 32767))
    b.flat[0] = signed_m31(-128)
    np.testing.assert_array_equal(Z.matmul_m31(a, b), oracle_matmul(a, b))
