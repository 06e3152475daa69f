"""Conv + ReLU + 2x2 max pool fused into one kernel (the conv's epilogue
pools its requantised outputs), bit-exact against the oracle's two ops.

The reference runs a separate max_pool2d pass after each conv
(psp-ml/src/kernels/naive.rs:98-132; examples/mnist-bench/src/generated.rs:
88-91,122-125).  A compiled model fuses a 3x3 conv with the 2x2 / stride-2
max pool after it on all three conv paths: the tensor-core implicit GEMM
(in_c % 16 == 0; the window's four pixels are lanes of one epilogue warp),
the row-streaming dense conv (32 -> 32, 32 -> 64, 64 -> 64; the window's rows
go to one epilogue set) and the small-channel dp4a conv (in_c in
{1, 2, 3, 4, 8}).  Shapes cover the
config 0 and config 2 layers, partial tiles (widths that are not powers of
two, N not a multiple of the tile), and a pool whose clamp is narrower than
the conv's, which must not fuse.
"""
import numpy as np
import pytest

from gpu_helpers import conv_desc, make_desc, random_quant
from pspml import capi

pytestmark = pytest.mark.gpu


def _model_parts(H, W, ci, co, zp_in, zp_out, conv_act, pool_act, seed):
    r = np.random.default_rng(seed)
    cd = conv_desc(capi.OP_CONV2D, H, W, ci, co, k=3, zp_in=zp_in, zp_out=zp_out, act=conv_act)
    pd = make_desc(kind=capi.OP_MAX_POOL2D, in_h=H, in_w=W, in_c=co, out_h=H // 2,
                   out_w=W // 2, out_c=co, kernel_h=2, kernel_w=2, stride_h=2, stride_w=2,
                   zp_in=zp_out, zp_out=zp_out, act_min=pool_act[0], act_max=pool_act[1])
    filt = r.integers(-127, 128, (co, 3, 3, ci)).astype(np.int8)
    bias, mult, shift = random_quant(r, co)
    parts = [filt.view(np.uint8).reshape(-1), bias.view(np.uint8), mult.view(np.uint8),
             shift.view(np.uint8)]
    offs, pos = [], 0
    for a in parts:
        offs.append(pos)
        pos += (a.size + 255) // 256 * 256
    blob = np.zeros(pos, np.uint8)
    for o, a in zip(offs, parts):
        blob[o:o + a.size] = a
    descs = np.concatenate([np.array(cd).reshape(1), np.array(pd).reshape(1)])
    descs["filter_off"][0], descs["bias_off"][0], descs["mult_off"][0], descs["shift_off"][0] = offs
    return descs, blob


def _run_chain(ctx, oracle_mod, descs, blob, batch, micro, seed):
    import torch
    r = np.random.default_rng(seed)
    H, W, ci = int(descs[0]["in_h"]), int(descs[0]["in_w"]), int(descs[0]["in_c"])
    x = r.integers(-128, 128, (batch, H, W, ci)).astype(np.int8)
    model = capi.Model(ctx, descs, blob, micro)
    fused = tuple(model.op_fused(i) for i in range(len(descs)))
    xi = torch.from_numpy(x.reshape(-1)).cuda()
    out = torch.full((batch * model.out_bytes,), 77, dtype=torch.int8, device="cuda")
    model.forward_device(xi.data_ptr(), out.data_ptr(), batch,
                         torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    ctx.check_device()
    model.close()
    return fused, out.cpu().numpy().reshape(batch, -1), oracle_mod.net_forward_s8(descs, blob, x)


def _run(ctx, oracle_mod, descs, blob, batch, micro, seed):
    import torch
    r = np.random.default_rng(seed)
    H, W, ci = int(descs[0]["in_h"]), int(descs[0]["in_w"]), int(descs[0]["in_c"])
    x = r.integers(-128, 128, (batch, H, W, ci)).astype(np.int8)
    model = capi.Model(ctx, descs, blob, micro)
    fused = (model.op_fused(0), model.op_fused(1))
    xi = torch.from_numpy(x.reshape(-1)).cuda()
    out = torch.full((batch * model.out_bytes,), 77, dtype=torch.int8, device="cuda")
    model.forward_device(xi.data_ptr(), out.data_ptr(), batch,
                         torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    ctx.check_device()
    model.close()
    got = out.cpu().numpy().reshape(batch, -1)
    want = oracle_mod.net_forward_s8(descs, blob, x)
    return fused, got, want


@pytest.mark.parametrize("H,W,ci,co,batch", [
    (64, 64, 16, 32, 3),     # tiles of 16 x 8 pixels over 64-pixel rows
    (32, 32, 64, 128, 5),    # 32-pixel rows
    (16, 16, 128, 128, 9),   # stage 2
    (8, 8, 256, 256, 17),    # stage 3 (two images per tile)
    (8, 8, 128, 192, 6),     # N = 192 in a 256-column tile (two epilogue groups, one half each)
    (6, 6, 32, 48, 7),       # 8-pixel tile rows with two invalid columns; N = 48 in a 64 tile
    (12, 20, 16, 32, 4),     # a second, mostly empty tile column
    (2, 2, 32, 16, 70),      # one pooled pixel per image
])
@pytest.mark.parametrize("act", ["relu", "none"])
def test_tensor_core_conv_pool(ctx, oracle_mod, H, W, ci, co, batch, act):
    # ReLU with zp_out -3 (clamp at the zero point: floor form), or no
    # activation with zp_out 5 (fast form).
    conv_act, zp_out = ((-3, 127), -3) if act == "relu" else ((-128, 127), 5)
    descs, blob = _model_parts(H, W, ci, co, -128, zp_out, conv_act, (-128, 127), H * W + co)
    fused, got, want = _run(ctx, oracle_mod, descs, blob, batch, batch, 1)
    assert fused == (1, 2)
    assert np.array_equal(got, want), f"{np.count_nonzero(got != want)} outputs differ"


@pytest.mark.parametrize("H,W,ci,co,batch", [
    (28, 28, 1, 8, 9),       # config 0 conv1
    (14, 14, 8, 16, 9),      # config 0 conv2
    (10, 6, 3, 12, 5),       # 12 channels in a 16-channel chunk
    (4, 4, 4, 4, 33),
])
def test_small_channel_conv_pool(ctx, oracle_mod, H, W, ci, co, batch):
    descs, blob = _model_parts(H, W, ci, co, -128, -128, (-128, 127), (-128, 127), ci * co)
    fused, got, want = _run(ctx, oracle_mod, descs, blob, batch, 4, 2)
    assert fused == (1, 2)
    assert np.array_equal(got, want), f"{np.count_nonzero(got != want)} outputs differ"


@pytest.mark.parametrize("ci", [8, 32])
def test_narrower_pool_clamp_is_not_fused(ctx, oracle_mod, ci):
    descs, blob = _model_parts(16, 16, ci, 32, -128, 0, (-128, 127), (-20, 100), 5)
    fused, got, want = _run(ctx, oracle_mod, descs, blob, 3, 3, 3)
    assert fused == (0, 0)
    assert np.array_equal(got, want)


@pytest.mark.parametrize("H,W,ci,co,zp_in,act", [
    (64, 64, 32, 32, -128, "relu"),   # config 2's s0b shape (two samples per tile)
    (64, 64, 32, 32, 3, "none"),      # s0b shape, fast requantisation form under the pool
    (48, 256, 32, 32, 0, "none"),     # two 128-pixel column tiles
    (12, 20, 32, 32, 21, "relu"),     # one sample per tile
    (7, 9, 32, 32, -128, "none"),     # odd sizes
    (32, 32, 32, 64, -128, "relu"),   # config 2's s1a shape (four samples per tile)
    (32, 32, 64, 64, -128, "relu"),   # config 2's s1b shape
    (16, 32, 64, 64, 40, "none"),     # four samples per tile, fast form under the pool
    (20, 48, 32, 64, 9, "none"),      # two samples per tile
    (9, 100, 64, 64, 0, "relu"),      # one sample per tile, odd height
    (5, 17, 64, 64, -7, "none"),
])
def test_row_streamed_dense_conv(ctx, oracle_mod, H, W, ci, co, zp_in, act):
    """3x3 stride-1 convs of 32 -> 32, 32 -> 64 and 64 -> 64 channels run on
    the row-streaming kernel with dense weight blocks (each input row loaded
    once); with even sizes the 2x2 max pool after the conv runs in its
    epilogue (a set of epilogue warps takes the window's two rows, lanes x
    and x ^ 1 its two columns)."""
    conv_act, zp_out = ((-3, 127), -3) if act == "relu" else ((-128, 127), 5)
    descs, blob = _model_parts(H, W, ci, co, zp_in, zp_out, conv_act, (-128, 127), H + W + ci)
    pooled = H % 2 == 0 and W % 2 == 0
    if not pooled:
        descs = descs[:1].copy()  # the conv alone
    fused, got, want = _run_chain(ctx, oracle_mod, descs, blob, 5, 5, 4)
    assert fused == ((1, 2) if pooled else (0,))
    assert np.array_equal(got, want), f"{np.count_nonzero(got != want)} outputs differ"
