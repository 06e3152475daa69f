"""Per-op parity on the B200: every int8 kernel through the C ABI against
the CPU oracle on the same seeded inputs.  Integer work: bit-exact."""
import numpy as np
import pytest

from gpu_helpers import conv_desc, make_desc, random_quant, run_op_gpu
from pspml import capi

pytestmark = pytest.mark.gpu


def _check(ctx, oracle_mod, d, batch, x, w=None, b=None, m=None, s=None):
    got = run_op_gpu(ctx, d, batch, x, w, b, m, s)
    want = oracle_mod.op_s8(d, batch, x, w, b, m, s)
    mism = np.flatnonzero(got != want)
    assert mism.size == 0, (f"{mism.size} of {want.size} differ; first at {mism[:5]}: "
                            f"got {got[mism[:5]]} want {want[mism[:5]]}")


# ------------------------------------------------------------------ FC (tcgen05)
@pytest.mark.parametrize("B,K,N", [
    (1, 512, 512), (7, 784, 10), (130, 256, 100), (257, 512, 3337), (64, 2048, 2048),
    (3, 96, 33), (129, 64, 256), (300, 32, 48), (2, 8192, 40),
    # Row lengths of every residue mod 4 above one 256-column tile (rows
    # not 4-byte aligned take the carried-word store path).
    (300, 64, 1002), (129, 128, 515),
    # Batches of 1-4 take the weight-streaming GEMV kernel.
    (4, 1024, 777), (1, 16, 3), (2, 4096, 4099)])
@pytest.mark.parametrize("mode", ["calibrated", "extreme"])
def test_fc_tensor_core(ctx, oracle_mod, B, K, N, mode):
    r = np.random.default_rng(B * 7 + K + N)
    x = r.integers(-128, 128, (B, K)).astype(np.int8)
    w = r.integers(-127, 128, (N, K)).astype(np.int8)
    b, m, s = random_quant(r, N, mode)
    d = make_desc(kind=capi.OP_FULLY_CONNECTED, in_h=1, in_w=1, in_c=K, out_h=1, out_w=1,
                  out_c=N, zp_in=-3, zp_out=5, act_min=5, act_max=127)
    _check(ctx, oracle_mod, d, B, x, w, b, m, s)


def test_fc_no_bias_full_range(ctx, oracle_mod):
    r = np.random.default_rng(5)
    B, K, N = 33, 160, 72
    x = r.integers(-128, 128, (B, K)).astype(np.int8)
    w = r.integers(-127, 128, (N, K)).astype(np.int8)
    _, m, s = random_quant(r, N)
    d = make_desc(kind=capi.OP_FULLY_CONNECTED, in_h=1, in_w=1, in_c=K, out_h=1, out_w=1,
                  out_c=N, zp_in=0, zp_out=-7)
    _check(ctx, oracle_mod, d, B, x, w, None, m, s)


@pytest.mark.parametrize("B,K,N", [(5, 100, 7), (3, 33, 129)])
def test_fc_cuda_core_odd_k(ctx, oracle_mod, B, K, N):
    r = np.random.default_rng(K)
    x = r.integers(-128, 128, (B, K)).astype(np.int8)
    w = r.integers(-127, 128, (N, K)).astype(np.int8)
    b, m, s = random_quant(r, N)
    d = make_desc(kind=capi.OP_FULLY_CONNECTED, in_h=1, in_w=1, in_c=K, out_h=1, out_w=1,
                  out_c=N, zp_in=-128, zp_out=0)
    _check(ctx, oracle_mod, d, B, x, w, b, m, s)


# -------------------------------------------------------- 1x1 conv (tcgen05)
@pytest.mark.parametrize("B,H,W,Ci,Co", [
    (2, 48, 256, 32, 64), (3, 12, 64, 128, 256), (1, 6, 32, 256, 512), (2, 5, 7, 64, 48),
    (2, 24, 128, 64, 128)])
def test_pointwise_conv(ctx, oracle_mod, B, H, W, Ci, Co):
    r = np.random.default_rng(H * W + Ci + Co)
    d = conv_desc(capi.OP_CONV2D, H, W, Ci, Co, k=1, zp_in=-128, zp_out=0)
    x = r.integers(-128, 128, (B, H, W, Ci)).astype(np.int8)
    w = r.integers(-127, 128, (Co, 1, 1, Ci)).astype(np.int8)
    b, m, s = random_quant(r, Co)
    _check(ctx, oracle_mod, d, B, x, w, b, m, s)


# ---------------------------------------------- 3x3 implicit GEMM (tcgen05)
@pytest.mark.parametrize("B,H,W,Ci,Co", [
    (2, 64, 64, 32, 32), (3, 16, 16, 64, 128), (5, 8, 8, 128, 256), (2, 28, 28, 32, 16),
    (3, 5, 7, 48, 40), (2, 32, 32, 32, 64), (2, 4, 4, 256, 256), (1, 1, 3, 32, 32)])
@pytest.mark.parametrize("zp_in", [-128, 0, 37])
def test_conv3x3_tensor_core(ctx, oracle_mod, B, H, W, Ci, Co, zp_in):
    r = np.random.default_rng(1000 + H * 31 + W + Ci * 3 + Co + zp_in)
    d = conv_desc(capi.OP_CONV2D, H, W, Ci, Co, k=3, zp_in=zp_in, zp_out=-128,
                  act=(-128, 127))
    x = r.integers(-128, 128, (B, H, W, Ci)).astype(np.int8)
    w = r.integers(-127, 128, (Co, 3, 3, Ci)).astype(np.int8)
    b, m, s = random_quant(r, Co)
    _check(ctx, oracle_mod, d, B, x, w, b, m, s)


def test_conv3x3_valid_padding(ctx, oracle_mod):
    r = np.random.default_rng(99)
    d = conv_desc(capi.OP_CONV2D, 10, 12, 32, 48, k=3, pad="valid", zp_in=-5, zp_out=3)
    x = r.integers(-128, 128, (3, 10, 12, 32)).astype(np.int8)
    w = r.integers(-127, 128, (48, 3, 3, 32)).astype(np.int8)
    b, m, s = random_quant(r, 48, "extreme")
    _check(ctx, oracle_mod, d, 3, x, w, b, m, s)


# ------------------------------------------------------- direct conv (CUDA cores)
@pytest.mark.parametrize("B,H,W,Ci,Co,k,stride", [
    (3, 28, 28, 1, 8, 3, 1), (2, 14, 14, 8, 16, 3, 1), (2, 64, 64, 3, 32, 3, 1),
    (2, 96, 512, 1, 32, 3, 2), (2, 9, 11, 5, 7, 3, 2), (2, 13, 13, 16, 24, 3, 2),
    (1, 10, 10, 4, 20, 5, 1)])
def test_conv_direct(ctx, oracle_mod, B, H, W, Ci, Co, k, stride):
    r = np.random.default_rng(H + W + Ci + Co + k + stride)
    d = conv_desc(capi.OP_CONV2D, H, W, Ci, Co, k=k, stride=stride, zp_in=-128, zp_out=-128)
    x = r.integers(-128, 128, (B, H, W, Ci)).astype(np.int8)
    w = r.integers(-127, 128, (Co, k, k, Ci)).astype(np.int8)
    b, m, s = random_quant(r, Co)
    _check(ctx, oracle_mod, d, B, x, w, b, m, s)


# 3x3 stride-1 convs with in_c in {1, 2, 3, 4, 8} run the 2x2-block kernel
# (one 4x4 input window per thread): odd output sizes leave partial blocks,
# Co = 36 a partial second channel chunk.
@pytest.mark.parametrize("B,H,W,Ci,Co", [
    (2, 7, 9, 2, 12), (3, 5, 11, 4, 8), (2, 13, 6, 8, 36), (4, 1, 1, 3, 4), (2, 9, 3, 1, 16)])
@pytest.mark.parametrize("zp_in,mode", [(-128, "calibrated"), (7, "calibrated"),
                                        (-3, "extreme")])
def test_small_conv_2x2_blocks(ctx, oracle_mod, B, H, W, Ci, Co, zp_in, mode):
    r = np.random.default_rng(1000 + 7 * H + W + 11 * Ci + Co + zp_in)
    d = conv_desc(capi.OP_CONV2D, H, W, Ci, Co, k=3, stride=1, zp_in=zp_in, zp_out=-5,
                  act=(-5, 127))
    x = r.integers(-128, 128, (B, H, W, Ci)).astype(np.int8)
    w = r.integers(-127, 128, (Co, 3, 3, Ci)).astype(np.int8)
    b, m, s = random_quant(r, Co, mode)
    _check(ctx, oracle_mod, d, B, x, w, b, m, s)


# ------------------------------------------------------------ depthwise conv
@pytest.mark.parametrize("B,H,W,C,stride", [
    (2, 48, 256, 32, 1), (2, 48, 256, 64, 2), (3, 12, 64, 256, 1), (2, 6, 32, 512, 1),
    (2, 7, 9, 12, 2), (1, 5, 5, 3, 1), (2, 24, 128, 128, 2)])
@pytest.mark.parametrize("zp_in", [-128, 0, 21])
def test_depthwise(ctx, oracle_mod, B, H, W, C, stride, zp_in):
    r = np.random.default_rng(1000 + H * W + C + stride + zp_in)
    d = conv_desc(capi.OP_DEPTHWISE_CONV2D, H, W, C, C, k=3, stride=stride, zp_in=zp_in,
                  zp_out=-128)
    x = r.integers(-128, 128, (B, H, W, C)).astype(np.int8)
    w = r.integers(-127, 128, (3, 3, C)).astype(np.int8)
    b, m, s = random_quant(r, C)
    _check(ctx, oracle_mod, d, B, x, w, b, m, s)


# ------------------------------------------------------------------ pooling
@pytest.mark.parametrize("B,H,W,C,act", [
    (3, 28, 28, 8, (-128, 127)), (2, 64, 64, 32, (-128, 127)), (2, 9, 9, 3, (-20, 60)),
    (2, 8, 8, 256, (-5, 5))])
def test_maxpool(ctx, oracle_mod, B, H, W, C, act):
    r = np.random.default_rng(H + C)
    d = make_desc(kind=capi.OP_MAX_POOL2D, in_h=H, in_w=W, in_c=C, out_h=H // 2, out_w=W // 2,
                  out_c=C, kernel_h=2, kernel_w=2, stride_h=2, stride_w=2, zp_in=-128,
                  zp_out=-128, act_min=act[0], act_max=act[1])
    x = r.integers(-128, 128, (B, H, W, C)).astype(np.int8)
    _check(ctx, oracle_mod, d, B, x)


@pytest.mark.parametrize("B,H,W,C", [(5, 6, 32, 512), (7, 4, 4, 256), (3, 3, 5, 7), (4, 5, 3, 12),
                                     (2, 7, 9, 48)])
def test_global_avgpool(ctx, oracle_mod, B, H, W, C):
    r = np.random.default_rng(H * W + C)
    d = make_desc(kind=capi.OP_AVERAGE_POOL2D, in_h=H, in_w=W, in_c=C, out_h=1, out_w=1,
                  out_c=C, kernel_h=H, kernel_w=W, stride_h=H, stride_w=W)
    x = r.integers(-128, 128, (B, H, W, C)).astype(np.int8)
    _check(ctx, oracle_mod, d, B, x)


@pytest.mark.parametrize("lo,hi,act", [(-128, -90, (-128, 127)), (90, 128, (-128, 127)),
                                       (-128, 128, (-40, 50))])
def test_global_avgpool_rounding_and_clamp(ctx, oracle_mod, lo, hi, act):
    # One-signed sums take each rounding branch; 39 pixels leave a remainder
    # after the eight-pixel steps of the global kernel.
    B, H, W, C = 6, 13, 3, 64
    r = np.random.default_rng(lo + 1000)
    d = make_desc(kind=capi.OP_AVERAGE_POOL2D, in_h=H, in_w=W, in_c=C, out_h=1, out_w=1,
                  out_c=C, kernel_h=H, kernel_w=W, stride_h=H, stride_w=W, act_min=act[0],
                  act_max=act[1])
    x = r.integers(lo, hi, (B, H, W, C)).astype(np.int8)
    _check(ctx, oracle_mod, d, B, x)


def test_empty_batch_is_a_no_op(ctx):
    d = make_desc(kind=capi.OP_MAX_POOL2D, in_h=4, in_w=4, in_c=16, out_h=2, out_w=2, out_c=16,
                  kernel_h=2, kernel_w=2, stride_h=2, stride_w=2)
    out = run_op_gpu(ctx, d, 0, np.zeros(16, np.int8))
    assert out.size == 0
