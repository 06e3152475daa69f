"""int8 oracle self-checks.  The reference has no int8 kernels, so the int8
oracle (TFLite reference semantics) is pinned by hand-computed known answers
of the fixed-point primitives and by agreement with float64 arithmetic."""
import math

import numpy as np
import pytest

from oracle import oracle as orc
from pspml import capi, netspec

I32_MIN, I32_MAX = -(1 << 31), (1 << 31) - 1


@pytest.mark.parametrize("a,b,expected", [
    (I32_MIN, I32_MIN, I32_MAX),          # the one saturating case
    (1 << 30, 1 << 30, 1 << 29),          # exact
    (1, 1 << 30, 1),                      # +0.5 rounds up
    (-1, 1 << 30, 0),                     # -0.5 rounds toward +inf (nudge 1-2^30)
    (3, 1 << 30, 2),                      # 1.5 -> 2
    (-3, 1 << 30, -1),                    # -1.5 -> -1
    (-1, (1 << 30) + 1, -1),              # just past -0.5
    (I32_MAX, I32_MAX, I32_MAX - 1),
    (I32_MIN, I32_MAX, -I32_MAX),
    (0, 12345, 0),
])
def test_srdhm_known(a, b, expected):
    assert orc.srdhm(a, b) == expected


@pytest.mark.parametrize("x,e,expected", [
    (5, 1, 3), (-5, 1, -3),               # ties away from zero
    (4, 1, 2), (-4, 1, -2),
    (7, 2, 2), (-7, 2, -2),
    (6, 2, 2), (-6, 2, -2),               # 1.5 -> 2, -1.5 -> -2
    (5, 2, 1), (-5, 2, -1),
    (123, 0, 123), (-123, 0, -123),
    (I32_MAX, 31, 1), (I32_MIN, 31, -1),
])
def test_rdbpot_known(x, e, expected):
    assert orc.rdbpot(x, e) == expected


def test_mbqm_known():
    assert orc.mbqm(100, 1 << 30, 0) == 50
    assert orc.mbqm(100, 1 << 30, -1) == 25
    assert orc.mbqm(101, 1 << 30, -1) == 26   # 50.5 -> 51, then 25.5 -> 26
    assert orc.mbqm(-101, 1 << 30, -1) == -25  # -50.5 -> -50, then -25
    assert orc.mbqm(3, 1 << 30, 2) == 6        # left shift first
    # the left shift wraps like int32: (2^30 << 2) == 0
    assert orc.mbqm(1 << 30, 1 << 30, 2) == 0


def _mbqm_float_ref(x, m, s):
    # exact rational value with the two roundings done in Python integers
    left, right = max(s, 0), max(-s, 0)
    a = ((x << left) + (1 << 31)) % (1 << 32) - (1 << 31)
    p = a * m
    h = (p + (1 << 30)) >> 31 if not (a == m == I32_MIN) else I32_MAX
    mask = (1 << right) - 1
    rem = h & mask
    thr = (mask >> 1) + (1 if h < 0 else 0)
    return (h >> right) + (1 if rem > thr else 0)


def test_mbqm_random_matches_closed_form():
    r = np.random.default_rng(7)
    for _ in range(20000):
        x = int(r.integers(-(1 << 28), 1 << 28))
        m = int(r.integers(1 << 30, 1 << 31))
        s = int(r.integers(-31, 3))
        assert orc.mbqm(x, m, s) == _mbqm_float_ref(x, m, s)


@pytest.mark.parametrize("real", [0.5, 0.25, 1.0, 0.75, 1e-3, 3.7e-5, 0.999999999, 2.5,
                                  0.0, 1e-20, 1e12])
def test_quantize_multiplier_matches_python(real):
    assert orc.quantize_multiplier(real) == netspec.quantize_multiplier(real)


def test_quantize_multiplier_known():
    assert orc.quantize_multiplier(0.5) == (1 << 30, 0)
    assert orc.quantize_multiplier(0.25) == (1 << 30, -1)
    assert orc.quantize_multiplier(1.0) == (1 << 30, 1)
    assert orc.quantize_multiplier(0.75) == (3 << 29, 0)
    assert orc.quantize_multiplier(0.0) == (0, 0)
    assert orc.quantize_multiplier(1e-20) == (0, 0)


def test_quantize_multiplier_represents_real():
    r = np.random.default_rng(3)
    for real in np.exp(r.uniform(math.log(1e-6), math.log(1.0), 500)):
        m, s = orc.quantize_multiplier(float(real))
        assert (1 << 30) <= m < (1 << 31)
        assert abs(m * 2.0 ** (s - 31) - real) <= real * 2.0 ** -30


def _desc(**kw):
    d = np.zeros(1, dtype=capi.OP_DESC_DTYPE)[0]
    base = dict(kind=capi.OP_FULLY_CONNECTED, in_h=1, in_w=1, in_c=1, out_h=1, out_w=1, out_c=1,
                kernel_h=1, kernel_w=1, stride_h=1, stride_w=1, act_min=-128, act_max=127,
                filter_off=-1, bias_off=-1, mult_off=-1, shift_off=-1)
    base.update(kw)
    for k, v in base.items():
        d[k] = v
    return d


def test_fc_int8_matches_float64_within_one_lsb():
    r = np.random.default_rng(11)
    B, K, N = 8, 96, 24
    zp_in, zp_out = -3, 5
    s_in, s_out = 0.02, 0.7
    ws = np.exp(r.uniform(math.log(1e-3), math.log(1e-1), N))
    x = r.integers(-128, 128, (B, K)).astype(np.int8)
    w = r.integers(-127, 128, (N, K)).astype(np.int8)
    b = r.integers(-4096, 4097, N).astype(np.int32)
    mult = np.zeros(N, np.int32)
    shift = np.zeros(N, np.int32)
    for c in range(N):
        mult[c], shift[c] = netspec.quantize_multiplier(s_in * ws[c] / s_out)
    d = _desc(in_c=K, out_c=N, zp_in=zp_in, zp_out=zp_out)
    got = orc.op_s8(d, B, x, w, b, mult, shift).reshape(B, N).astype(np.int32)
    acc = (x.astype(np.float64) - zp_in) @ w.astype(np.float64).T + b
    real = acc * (s_in * ws)
    want = np.clip(np.rint(real / s_out) + zp_out, -128, 127)
    assert np.max(np.abs(got - want)) <= 1


def test_conv_padding_is_real_zero():
    # A conv over a constant input equal to the zero point gives bias only,
    # also at the borders: padded taps contribute nothing.
    H = W = 5
    C, CO = 3, 4
    d = _desc(kind=capi.OP_CONV2D, in_h=H, in_w=W, in_c=C, out_h=H, out_w=W, out_c=CO,
              kernel_h=3, kernel_w=3, pad_top=1, pad_left=1, pad_bottom=1, pad_right=1,
              zp_in=-77, zp_out=0)
    x = np.full((1, H, W, C), -77, np.int8)
    w = np.random.default_rng(1).integers(-127, 128, (CO, 3, 3, C)).astype(np.int8)
    b = np.array([100, -200, 300, -400], np.int32)
    mult = np.full(CO, 1 << 30, np.int32)
    shift = np.zeros(CO, np.int32)
    y = orc.op_s8(d, 1, x, w, b, mult, shift).reshape(H, W, CO)
    assert np.all(y == np.clip(np.array([50, -100, 127, -128]), -128, 127))


def test_avgpool_rounding_half_away():
    d = _desc(kind=capi.OP_AVERAGE_POOL2D, in_h=1, in_w=2, in_c=1, out_h=1, out_w=1, out_c=1,
              kernel_h=1, kernel_w=2, stride_h=1, stride_w=2)
    for pair, want in (((1, 2), 2), ((-1, -2), -2), ((3, 4), 4), ((-3, -4), -4), ((2, 2), 2)):
        assert orc.op_s8(d, 1, np.array(pair, np.int8))[0] == want


def test_maxpool_clamps_to_activation_range():
    d = _desc(kind=capi.OP_MAX_POOL2D, in_h=2, in_w=2, in_c=1, out_h=1, out_w=1, out_c=1,
              kernel_h=2, kernel_w=2, stride_h=2, stride_w=2, act_min=-10, act_max=20)
    assert orc.op_s8(d, 1, np.array([-50, -40, -30, -20], np.int8))[0] == -10
    assert orc.op_s8(d, 1, np.array([50, -40, -30, -20], np.int8))[0] == 20
