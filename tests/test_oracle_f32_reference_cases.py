"""The oracle's f32 kernels against the reference's own known-answer tests
(psp-ml/src/bin/test-kernels.rs:47-390) and SAME-padding unit tests
(cargo-psp-ml/src/parse/tflite/lowering.rs:366-420).  This pins the f32
oracle to the reference."""
import numpy as np
import pytest

from golden import ref_kernel_cases as R
from oracle import oracle as orc


def approx_eq(a, b):
    a = np.asarray(a, dtype=np.float32).reshape(-1)
    b = np.asarray(b, dtype=np.float32).reshape(-1)
    return a.shape == b.shape and bool(np.all(np.abs(a - b) <= R.EPS))


def test_relu():
    assert approx_eq(orc.f32_relu(R.RELU_IN), R.RELU_EXPECTED)


def test_relu_keeps_negative_zero():
    # `if x < 0.0 { x = 0.0 }` leaves -0.0 untouched (mod.rs:347-364)
    y = orc.f32_relu(np.array([-0.0], dtype=np.float32))
    assert np.signbit(y[0])


def test_bias_add():
    assert approx_eq(orc.f32_bias_add(R.BIAS_ADD_DATA, R.BIAS_ADD_BIAS, 3, 4), R.BIAS_ADD_EXPECTED)


def test_matmul_bt_identity():
    assert approx_eq(orc.f32_matmul_bt(R.MM_ID_A, R.MM_ID_B, 4, 4, 4), R.MM_ID_A)


def test_matmul_bt_known():
    assert approx_eq(orc.f32_matmul_bt(R.MM_KNOWN_A, R.MM_KNOWN_B, 4, 8, 4), R.MM_KNOWN_EXPECTED)


def test_matmul_bt_non_aligned():
    assert approx_eq(orc.f32_matmul_bt(R.MM_NA_A, R.MM_NA_B, 5, 6, 3), R.mm_na_expected())


def test_matmul_bt_tiled():
    ref = orc.f32_matmul_bt(R.MM_TILED_A, R.MM_TILED_B, 8, 8, 4)
    assert approx_eq(orc.f32_matmul_bt_tiled(R.MM_TILED_A, R.MM_TILED_B, 2, 2, 1), ref)


def test_matmul_bt_tiled_large():
    ref = orc.f32_matmul_bt(R.MM_TL_A, R.MM_TL_B, 16, 20, 8)
    assert approx_eq(orc.f32_matmul_bt_tiled(R.MM_TL_A, R.MM_TL_B, 4, 5, 2), ref)


def test_im2col_simple():
    col = orc.f32_im2col(R.IM2COL_IN, (1, 4, 4, 1), (3, 3), (1, 1), (0, 0), (2, 2))
    assert approx_eq(col[0:9], R.IM2COL_SIMPLE_ROW0)
    assert approx_eq(col[9:18], R.IM2COL_SIMPLE_ROW1)


def test_im2col_with_padding():
    col = orc.f32_im2col(R.IM2COL_IN, (1, 4, 4, 1), (3, 3), (1, 1), (1, 1), (4, 4))
    assert approx_eq(col[0:9], R.IM2COL_PAD_ROW0)


def test_im2col_padded_vs_im2col():
    ref = orc.f32_im2col(R.IM2COL_PVI_IN, (1, 4, 4, 2), (3, 3), (1, 1), (1, 1), (4, 4))
    pad = orc.f32_im2col_padded(R.IM2COL_PVI_IN, (1, 4, 4, 2), (3, 3), (1, 1), (4, 4))
    for row in range(16):
        assert approx_eq(ref[row * 18:(row + 1) * 18], pad[row * 20:row * 20 + 18])
        assert pad[row * 20 + 18] == 0.0 and pad[row * 20 + 19] == 0.0


def test_im2col_padded_leaves_pad_columns():
    # the pad columns are never written (mod.rs:421-422): the caller zeroes them
    pad = orc.f32_im2col_padded(R.IM2COL_PVI_IN, (1, 4, 4, 2), (3, 3), (1, 1), (4, 4), fill=7.0)
    assert np.all(pad.reshape(16, 20)[:, 18:] == 7.0)


def test_conv2d_via_im2col_vs_naive():
    ci, co, h, w, kh, kw = 2, 4, 6, 6, 3, 3
    naive = orc.f32_conv2d(R.CONV_IN, (1, h, w, ci), R.CONV_FILTER, (co, kh, kw, ci), R.CONV_BIAS,
                           (1, 1), (1, 1), (1, h, w, co), relu=True)
    col = orc.f32_im2col_padded(R.CONV_IN, (1, h, w, ci), (kh, kw), (1, 1), (h, w))
    k, kp = 18, 20
    wpad = np.zeros(co * kp, dtype=np.float32)
    for r in range(co):
        wpad[r * kp:r * kp + k] = R.CONV_FILTER[r * k:(r + 1) * k]
    out = orc.f32_matmul_bt_tiled(col, wpad, 36 // 4, kp // 4, co // 4)
    out = orc.f32_relu(orc.f32_bias_add(out, R.CONV_BIAS, 36, co))
    assert approx_eq(out, naive)


@pytest.mark.parametrize("args,expected", R.SAME_PADDING_CASES)
def test_same_padding(args, expected):
    assert orc.same_padding(*args) == expected


def test_same_padding_rectangular():
    args, (sum_h, sum_w) = R.SAME_PADDING_RECT
    t, b, l, r = orc.same_padding(*args)
    assert t + b == sum_h and l + r == sum_w


def test_max_pool_and_fc_small():
    x = np.arange(16, dtype=np.float32) - 8
    y = orc.f32_max_pool2d(x, (1, 4, 4, 1), (2, 2), (2, 2), (1, 2, 2, 1))
    assert approx_eq(y, [-3, -1, 5, 7])
    w = np.array([1, 0, -1, 2, 2, 2], dtype=np.float32)
    b = np.array([0.5, -100.0], dtype=np.float32)
    xin = np.array([1, 2, 3], dtype=np.float32)
    assert approx_eq(orc.f32_fully_connected(xin, 3, w, b, 2), [-1.5, -88.0])
    assert approx_eq(orc.f32_fully_connected(xin, 3, w, b, 2, relu=True), [0.0, 0.0])
