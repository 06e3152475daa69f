"""Known-answer cases of the reference's kernel test harness, restated.

Source: psp-ml/src/bin/test-kernels.rs (saifk00/psp-ml), absolute tolerance
EPS = 1e-4 (test-kernels.rs:19-32); last recorded run 11/11 passed
(psp-ml/test-results.json).  Inputs follow the formulas of each test; the
expected arrays are the literal ones the reference asserts.  The same-padding
values are the reference's unit tests at
cargo-psp-ml/src/parse/tflite/lowering.rs:366-420.
"""
import numpy as np

EPS = 1e-4

# test_relu, test-kernels.rs:47-52
RELU_IN = np.array([-2.0, -1.0, 0.0, 1.0, 2.0, 3.0, -0.5, 0.5], dtype=np.float32)
RELU_EXPECTED = np.array([0.0, 0.0, 0.0, 1.0, 2.0, 3.0, 0.0, 0.5], dtype=np.float32)

# test_bias_add, test-kernels.rs:54-69
BIAS_ADD_DATA = np.array([1, 2, 3, 4, 5, 6, 7, 8, 9, 10, 11, 12], dtype=np.float32)
BIAS_ADD_BIAS = np.array([0.1, 0.2, 0.3, 0.4], dtype=np.float32)
BIAS_ADD_EXPECTED = np.array(
    [1.1, 2.2, 3.3, 4.4, 5.1, 6.2, 7.3, 8.4, 9.1, 10.2, 11.3, 12.4], dtype=np.float32)

# test_matmul_bt_identity, test-kernels.rs:71-87: A[4,4] @ I^T = A
MM_ID_A = np.arange(1, 17, dtype=np.float32)
MM_ID_B = np.eye(4, dtype=np.float32).reshape(-1)

# test_matmul_bt_known, test-kernels.rs:89-138: A[4,8] @ B[4,8]^T
MM_KNOWN_A = np.array([
    1, 2, 0, 0, 0, 0, 0, 0,
    0, 0, 3, 4, 0, 0, 0, 0,
    0, 0, 0, 0, 5, 6, 0, 0,
    0, 0, 0, 0, 0, 0, 7, 8], dtype=np.float32)
MM_KNOWN_B = np.array([
    1, 1, 1, 1, 0, 0, 0, 0,
    0, 0, 0, 0, 1, 1, 1, 1,
    1, 0, 0, 0, 0, 0, 0, 1,
    0, 1, 0, 0, 0, 0, 1, 0], dtype=np.float32)
MM_KNOWN_EXPECTED = np.array([
    3, 0, 1, 2,
    7, 0, 0, 0,
    0, 11, 0, 0,
    0, 15, 8, 7], dtype=np.float32)

# test_matmul_bt_non_aligned, test-kernels.rs:140-165: A[5,6] @ B[3,6]^T,
# expected by a sequential triple loop.
MM_NA_A = np.array([
    1.0, 2.0, 3.0, 4.0, 5.0, 6.0,
    7.0, 8.0, 9.0, 10.0, 11.0, 12.0,
    0.5, 1.5, 2.5, 3.5, 4.5, 5.5,
    -1.0, -2.0, -3.0, -4.0, -5.0, -6.0,
    0.1, 0.2, 0.3, 0.4, 0.5, 0.6], dtype=np.float32)
MM_NA_B = np.array([
    1.0, 0.0, 1.0, 0.0, 1.0, 0.0,
    0.0, 1.0, 0.0, 1.0, 0.0, 1.0,
    1.0, 1.0, 0.0, 0.0, 1.0, 1.0], dtype=np.float32)


def mm_na_expected() -> np.ndarray:
    out = np.zeros(15, dtype=np.float32)
    for i in range(5):
        for j in range(3):
            s = np.float32(0.0)
            for k in range(6):
                s = np.float32(s + np.float32(MM_NA_A[i * 6 + k] * MM_NA_B[j * 6 + k]))
            out[i * 3 + j] = s
    return out


# test_matmul_bt_tiled, test-kernels.rs:167-182: A[8,8], B[4,8]; tiles (2,2,1)
MM_TILED_A = (np.arange(64, dtype=np.float32) * np.float32(0.1)).astype(np.float32)
MM_TILED_B = (np.arange(32, dtype=np.float32) * np.float32(0.05) + np.float32(0.01)).astype(np.float32)

# test_matmul_bt_tiled_large, test-kernels.rs:184-200: A[16,20], B[8,20]; tiles (4,5,2)
MM_TL_A = ((np.arange(320) % 17).astype(np.float32) * np.float32(0.1) - np.float32(0.8)).astype(np.float32)
MM_TL_B = ((np.arange(160) % 13).astype(np.float32) * np.float32(0.07) - np.float32(0.4)).astype(np.float32)

# test_im2col_simple, test-kernels.rs:202-224: [1,4,4,1], 3x3, stride 1, no pad
IM2COL_IN = np.arange(1, 17, dtype=np.float32)
IM2COL_SIMPLE_ROW0 = np.array([1, 2, 3, 5, 6, 7, 9, 10, 11], dtype=np.float32)
IM2COL_SIMPLE_ROW1 = np.array([2, 3, 4, 6, 7, 8, 10, 11, 12], dtype=np.float32)

# test_im2col_with_padding, test-kernels.rs:226-254: pad [1,1]
IM2COL_PAD_ROW0 = np.array([0, 0, 0, 0, 1, 2, 0, 5, 6], dtype=np.float32)

# test_im2col_padded_vs_im2col, test-kernels.rs:256-299: [1,4,4,2], 3x3, pad 1
IM2COL_PVI_IN = (np.arange(32, dtype=np.float32) * np.float32(0.1) + np.float32(0.05)).astype(np.float32)

# test_conv2d_via_im2col_vs_naive, test-kernels.rs:301-390: [1,6,6,2] x [4,3,3,2]
CONV_IN = ((np.arange(72) % 11).astype(np.float32) * np.float32(0.1) - np.float32(0.5)).astype(np.float32)
CONV_FILTER = ((np.arange(72) % 7).astype(np.float32) * np.float32(0.05) - np.float32(0.15)).astype(np.float32)
CONV_BIAS = np.array([0.1, -0.2, 0.05, 0.3], dtype=np.float32)

# compute_same_padding unit tests, lowering.rs:366-420:
# (in_h, in_w, k_h, k_w, s_h, s_w) -> (top, bottom, left, right)
SAME_PADDING_CASES = [
    ((28, 28, 3, 3, 1, 1), (1, 1, 1, 1)),
    ((28, 28, 5, 5, 1, 1), (2, 2, 2, 2)),
    ((28, 28, 3, 3, 2, 2), (0, 1, 0, 1)),
    ((7, 7, 3, 3, 2, 2), (1, 1, 1, 1)),
    ((4, 4, 1, 1, 1, 1), (0, 0, 0, 0)),
]
# test_same_padding_rectangular: only the sums are asserted.
SAME_PADDING_RECT = ((28, 14, 3, 5, 1, 1), (2, 4))
