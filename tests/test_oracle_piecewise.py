"""Oracle piecewise-linear activation (no GPU): the integer activation functions and
segment coefficients, and prove -> verifier replay with identical transcripts,
tamper rejection."""
import numpy as np
import pytest

import oracle_lib as O
from helpers import int_matrix_m31, random_qm31, uniform_m31

P = (1 << 31) - 1
HALF = P // 2


def sigmoid_int(x, scale=HALF):
    def tdiv(a, b):
        q = abs(a) // abs(b)
        return q if (a >= 0) == (b > 0) else -q
    x5, x25 = scale * 5, tdiv(scale * 5, 2)
    if x <= -x5:
        return 0
    if x >= x5:
        return scale
    if x <= -x25:
        return tdiv((x + x5) * 28, tdiv(1000 * (x5 - x25), scale))
    if x >= x25:
        return tdiv(scale * 93, 100) + tdiv((x - x25) * 7, tdiv(100 * (x5 - x25), scale))
    return tdiv(scale, 2) + tdiv(x, 4)


@pytest.mark.parametrize("v", [0, 1, 5, 1 << 20, HALF, HALF + 1, P - 1, P - 12345, 1 << 30, 123456789])
def test_activation_integer_silu_sigmoid(v):
    s = v if v <= HALF else v - P

    def tdiv(a, b):
        q = abs(a) // abs(b)
        return q if (a >= 0) == (b > 0) else -q
    assert O.lib().orc_activation_integer(2, v) == sigmoid_int(s) % P
    assert O.lib().orc_activation_integer(4, v) == tdiv(s * sigmoid_int(s), HALF) % P
    assert O.lib().orc_activation_integer(0, v) == (s if s > 0 else 0)


def test_piecewise_coeffs_interpolate_segment_ends():
    for tag in range(1, 6):
        sl, ic = O.piecewise_coeffs(tag)
        for i in range(16):
            xs = i << 27
            xe = P - 1 if i == 15 else ((i + 1) << 27) - 1
            for x in (xs, xe):
                assert (int(sl[i]) * x + int(ic[i])) % P == O.lib().orc_activation_integer(tag - 1, x)


@pytest.mark.parametrize("rows,cols,tag", [(1, 2, 5), (1, 8, 5), (2, 3, 2), (4, 16, 3), (3, 5, 4), (8, 32, 5)])
def test_piecewise_roundtrip(rows, cols, tag):
    x = uniform_m31(rows * cols, rows + cols).reshape(rows, cols) if tag != 2 else \
        int_matrix_m31(rows, cols, 5, bound=1 << 29)
    rng = np.random.default_rng(rows * 3 + cols)
    nv = (rows - 1).bit_length() + (cols - 1).bit_length()
    point, value = random_qm31(nv, rng), random_qm31(1, rng)[0]
    ch = O.new_channel()
    rc, raw, ie, nxt = O.reduce_activation_piecewise(x, tag, point, value, ch)
    assert rc == 0 and nxt.shape == (nv, 4)
    vch = O.new_channel()
    ok, ie2 = O.verify_activation_piecewise(raw, point, value, vch)
    assert ok and (ie == ie2).all() and vch.digest_int() == ch.digest_int()
    bad = raw.copy()
    bad[4 * 16] ^= 1  # round 0, c0
    assert not O.verify_activation_piecewise(bad, point, value, O.new_channel())[0]
