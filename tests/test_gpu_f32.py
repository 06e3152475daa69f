"""The f32 path of the reference's own MNIST CNN on the B200, bit-exact.

The reference's generated code runs every conv as im2col_padded ->
matmul_bt_tiled -> bias_add -> relu and calls naive::max_pool2d and
naive::fully_connected[_relu] (psp-ml/src/kernels/mod.rs:176-479,
psp-ml/src/kernels/naive.rs:13-184).  The kernels behind
pspml_conv2d_f32 / pspml_max_pool2d_f32 / pspml_fully_connected_f32 follow
the same summation orders with separately rounded products and sums, so the
outputs equal the oracle's restatement of those functions exactly.
"""
import ctypes

import numpy as np
import pytest

from gpu_helpers import make_desc
from pspml import capi

pytestmark = pytest.mark.gpu

F32_RELU = capi.F32_RELU
F32_GEMM = capi.F32_GEMM_ORDER


def _same_pad(n, k):
    total = max(k - 1, 0)
    return total // 2, total - total // 2


def conv_f32_desc(H, W, Ci, Co, k, flags):
    pt, pb = _same_pad(H, k)
    pl, pr = _same_pad(W, k)
    return make_desc(kind=capi.OP_CONV2D, in_h=H, in_w=W, in_c=Ci, out_h=H, out_w=W, out_c=Co,
                     kernel_h=k, kernel_w=k, pad_top=pt, pad_left=pl, pad_bottom=pb,
                     pad_right=pr, flags=flags)


def pool_f32_desc(H, W, C):
    return make_desc(kind=capi.OP_MAX_POOL2D, in_h=H, in_w=W, in_c=C, out_h=H // 2,
                     out_w=W // 2, out_c=C, kernel_h=2, kernel_w=2, stride_h=2, stride_w=2)


def fc_f32_desc(K, N, flags):
    return make_desc(kind=capi.OP_FULLY_CONNECTED, in_h=1, in_w=1, in_c=K, out_h=1, out_w=1,
                     out_c=N, flags=flags)


def _gpu(ctx, fn, d, batch, x, *weights):
    import torch
    xt = torch.from_numpy(np.ascontiguousarray(x, np.float32).reshape(-1)).cuda()
    ws = [None if a is None else torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda()
          for a in weights]
    n_out = batch * int(d["out_h"]) * int(d["out_w"]) * int(d["out_c"])
    out = torch.full((n_out,), float("nan"), dtype=torch.float32, device="cuda")
    ds = capi.desc_struct(d)
    ptrs = [ctypes.c_void_p(w.data_ptr()) if w is not None else None for w in ws]
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    capi.call(fn, ctx.handle, ctypes.byref(ds), batch, ctypes.c_void_p(xt.data_ptr()), *ptrs,
              ctypes.c_void_p(out.data_ptr()), stream)
    torch.cuda.synchronize()
    ctx.check_device()
    return out.cpu().numpy()


def oracle_conv(oracle_mod, d, batch, x, w, b):
    """The oracle's reference restatement in the order the flags select."""
    H, W, Ci = int(d["in_h"]), int(d["in_w"]), int(d["in_c"])
    Co, k = int(d["out_c"]), int(d["kernel_h"])
    pad = (int(d["pad_top"]), int(d["pad_left"]))
    flags = int(d["flags"])
    relu = bool(flags & F32_RELU)
    if flags & F32_GEMM:
        K = k * k * Ci
        kp = (K + 3) // 4 * 4
        col = oracle_mod.f32_im2col_padded(x, (batch, H, W, Ci), (k, k), pad, (H, W))
        wp = np.zeros((Co + 3) // 4 * 4 * kp, np.float32)
        wp.reshape(-1, kp)[:Co, :K] = w.reshape(Co, K)
        rows = batch * H * W
        colp = np.zeros((rows + 3) // 4 * 4 * kp, np.float32)
        colp[:rows * kp] = col
        c = oracle_mod.f32_matmul_bt_tiled(colp, wp, (rows + 3) // 4, kp // 4, (Co + 3) // 4)
        c = c.reshape(-1, (Co + 3) // 4 * 4)[:rows, :Co].copy().reshape(-1)
        c = oracle_mod.f32_bias_add(c, b, rows, Co)
        return oracle_mod.f32_relu(c) if relu else c
    return oracle_mod.f32_conv2d(x, (batch, H, W, Ci), w, (Co, k, k, Ci), b, (1, 1), pad,
                                 (batch, H, W, Co), relu=relu)


@pytest.mark.parametrize("B,H,W,Ci,Co,k,flags", [
    (3, 28, 28, 1, 8, 5, F32_RELU | F32_GEMM),   # MNIST conv 1 as the reference runs it
    (2, 14, 14, 8, 16, 5, F32_RELU | F32_GEMM),  # MNIST conv 2
    (2, 9, 7, 3, 5, 3, F32_GEMM),                # K = 27, padded to 28
    (2, 14, 14, 8, 16, 5, F32_RELU),             # naive::conv2d_relu order
    (1, 6, 5, 2, 3, 3, 0),
])
def test_conv2d_f32(ctx, oracle_mod, B, H, W, Ci, Co, k, flags):
    r = np.random.default_rng(500 + H * W + Ci + Co + flags)
    d = conv_f32_desc(H, W, Ci, Co, k, flags)
    x = r.standard_normal(B * H * W * Ci).astype(np.float32)
    w = (r.standard_normal(Co * k * k * Ci) * 0.2).astype(np.float32)
    b = (r.standard_normal(Co) * 0.1).astype(np.float32)
    got = _gpu(ctx, "pspml_conv2d_f32", d, B, x, w, b)
    want = oracle_conv(oracle_mod, d, B, x, w, b)
    assert np.array_equal(got, want)


def test_max_pool2d_f32(ctx, oracle_mod):
    r = np.random.default_rng(9)
    B, H, W, C = 3, 28, 28, 8
    d = pool_f32_desc(H, W, C)
    x = r.standard_normal(B * H * W * C).astype(np.float32)
    got = _gpu(ctx, "pspml_max_pool2d_f32", d, B, x)
    want = oracle_mod.f32_max_pool2d(x, (B, H, W, C), (2, 2), (2, 2), (B, H // 2, W // 2, C))
    assert np.array_equal(got, want)


@pytest.mark.parametrize("B,K,N,flags", [(5, 784, 64, F32_RELU), (5, 64, 10, 0), (1, 3, 2, 0)])
def test_fully_connected_f32(ctx, oracle_mod, B, K, N, flags):
    r = np.random.default_rng(K + N)
    d = fc_f32_desc(K, N, flags)
    x = r.standard_normal(B * K).astype(np.float32)
    w = (r.standard_normal(N * K) * 0.05).astype(np.float32)
    b = r.standard_normal(N).astype(np.float32)
    got = _gpu(ctx, "pspml_fully_connected_f32", d, B, x, w, b).reshape(B, N)
    for i in range(B):
        want = oracle_mod.f32_fully_connected(x[i * K:(i + 1) * K], K, w, b, N,
                                              relu=bool(flags & F32_RELU))
        assert np.array_equal(got[i], want)


def test_mnist_cnn_f32_network(ctx, oracle_mod):
    """The reference's MNIST CNN architecture (conv 5x5 1->8 SAME ReLU,
    max pool, conv 5x5 8->16 SAME ReLU, max pool, reshape, FC 784->64 ReLU,
    FC 64->10) with synthetic weights, op by op on the GPU against the
    oracle chain."""
    r = np.random.default_rng(2024)
    B = 17
    x = r.random(B * 28 * 28).astype(np.float32)
    w1 = (r.standard_normal(8 * 25) * 0.3).astype(np.float32)
    b1 = (r.standard_normal(8) * 0.1).astype(np.float32)
    w2 = (r.standard_normal(16 * 25 * 8) * 0.1).astype(np.float32)
    b2 = (r.standard_normal(16) * 0.1).astype(np.float32)
    w3 = (r.standard_normal(64 * 784) * 0.05).astype(np.float32)
    b3 = (r.standard_normal(64) * 0.1).astype(np.float32)
    w4 = (r.standard_normal(10 * 64) * 0.2).astype(np.float32)
    b4 = (r.standard_normal(10) * 0.1).astype(np.float32)
    c1 = conv_f32_desc(28, 28, 1, 8, 5, F32_RELU | F32_GEMM)
    p1 = pool_f32_desc(28, 28, 8)
    c2 = conv_f32_desc(14, 14, 8, 16, 5, F32_RELU | F32_GEMM)
    p2 = pool_f32_desc(14, 14, 16)
    f1 = fc_f32_desc(784, 64, F32_RELU)
    f2 = fc_f32_desc(64, 10, 0)
    g = _gpu(ctx, "pspml_conv2d_f32", c1, B, x, w1, b1)
    g = _gpu(ctx, "pspml_max_pool2d_f32", p1, B, g)
    g = _gpu(ctx, "pspml_conv2d_f32", c2, B, g, w2, b2)
    g = _gpu(ctx, "pspml_max_pool2d_f32", p2, B, g)
    g = _gpu(ctx, "pspml_fully_connected_f32", f1, B, g, w3, b3)
    g = _gpu(ctx, "pspml_fully_connected_f32", f2, B, g, w4, b4).reshape(B, 10)
    o = oracle_conv(oracle_mod, c1, B, x, w1, b1)
    o = oracle_mod.f32_max_pool2d(o, (B, 28, 28, 8), (2, 2), (2, 2), (B, 14, 14, 8))
    o = oracle_conv(oracle_mod, c2, B, o, w2, b2)
    o = oracle_mod.f32_max_pool2d(o, (B, 14, 14, 16), (2, 2), (2, 2), (B, 7, 7, 16))
    for i in range(B):
        h = oracle_mod.f32_fully_connected(o[i * 784:(i + 1) * 784], 784, w3, b3, 64, relu=True)
        logits = oracle_mod.f32_fully_connected(h, 64, w4, b4, 10)
        assert np.array_equal(g[i], logits)


def test_reference_mnist_model_weights_f32(ctx, oracle_mod):
    """The reference's own MNIST model (mnist_cnn.tflite's trained weights,
    tests/golden/mnist_cnn_f32.npz made by make_mnist_f32_fixture.py) on the
    GPU, op by op, bit-identical to the oracle chain.  Inputs are seeded
    u8 pixels / 255, the reference's input conversion (main.rs:25-32)."""
    from pathlib import Path
    fx = np.load(Path(__file__).resolve().parent / "golden" / "mnist_cnn_f32.npz")
    r = np.random.default_rng(77)
    B = 33
    x = (r.integers(0, 256, B * 28 * 28).astype(np.float32) / np.float32(255.0))
    w1, b1 = fx["conv1_w"].reshape(-1), fx["conv1_b"]
    w2, b2 = fx["conv2_w"].reshape(-1), fx["conv2_b"]
    w3, b3 = fx["fc1_w"].reshape(-1), fx["fc1_b"]
    w4, b4 = fx["fc2_w"].reshape(-1), fx["fc2_b"]
    assert fx["conv1_relu"] and fx["conv2_relu"] and fx["fc1_relu"] and not fx["fc2_relu"]
    c1 = conv_f32_desc(28, 28, 1, 8, 5, F32_RELU | F32_GEMM)
    p1 = pool_f32_desc(28, 28, 8)
    c2 = conv_f32_desc(14, 14, 8, 16, 5, F32_RELU | F32_GEMM)
    p2 = pool_f32_desc(14, 14, 16)
    f1 = fc_f32_desc(784, 64, F32_RELU)
    f2 = fc_f32_desc(64, 10, 0)
    g = _gpu(ctx, "pspml_conv2d_f32", c1, B, x, w1, b1)
    g = _gpu(ctx, "pspml_max_pool2d_f32", p1, B, g)
    g = _gpu(ctx, "pspml_conv2d_f32", c2, B, g, w2, b2)
    g = _gpu(ctx, "pspml_max_pool2d_f32", p2, B, g)
    g = _gpu(ctx, "pspml_fully_connected_f32", f1, B, g, w3, b3)
    g = _gpu(ctx, "pspml_fully_connected_f32", f2, B, g, w4, b4).reshape(B, 10)
    o = oracle_conv(oracle_mod, c1, B, x, w1, b1)
    o = oracle_mod.f32_max_pool2d(o, (B, 28, 28, 8), (2, 2), (2, 2), (B, 14, 14, 8))
    o = oracle_conv(oracle_mod, c2, B, o, w2, b2)
    o = oracle_mod.f32_max_pool2d(o, (B, 14, 14, 16), (2, 2), (2, 2), (B, 7, 7, 16))
    for i in range(B):
        h = oracle_mod.f32_fully_connected(o[i * 784:(i + 1) * 784], 784, w3, b3, 64, relu=True)
        logits = oracle_mod.f32_fully_connected(h, 64, w4, b4, 10)
        assert np.array_equal(g[i], logits)
    assert np.all(np.isfinite(g))
