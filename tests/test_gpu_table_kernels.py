"""Layer-level parity of the constant-table kernels on the B200.

A compiled model builds a host requantisation table for every op whose
channels all take the fast requant form, and then runs the GEMM and the
tensor-core depthwise kernel with compile-time table offsets (border
classes as bias differences, 256-row GEMM tiles for narrow outputs).  These
tests run single ops through that path and compare every output byte with
the oracle (the whole-network tests only see the logits, after global
average pooling)."""
import zlib

import numpy as np
import pytest

from gpu_helpers import conv_desc, make_desc, random_quant, run_chain_model, run_op_model
from pspml import capi

pytestmark = pytest.mark.gpu


def _check(got, want):
    mism = np.flatnonzero(got != want)
    assert mism.size == 0, (f"{mism.size} of {want.size} differ; first at {mism[:5]}: "
                            f"got {got[mism[:5]]} want {want[mism[:5]]}")


@pytest.mark.parametrize("B,H,W,C,zp_in,act", [
    (2, 5, 256, 32, -128, (-128, 127)),
    (3, 4, 128, 64, 0, (-128, 127)),
    (2, 3, 200, 128, 7, (-20, 90)),      # partial second tile, clamp
    (1, 6, 384, 96, -3, (-128, 127)),    # three channel groups, three tiles
    (2, 1, 130, 32, 5, (0, 127)),        # one row: every tile row is a border row
])
def test_depthwise_static_table(ctx, oracle_mod, B, H, W, C, zp_in, act):
    r = np.random.default_rng(7000 + H * W + C)
    d = conv_desc(capi.OP_DEPTHWISE_CONV2D, H, W, C, C, k=3, stride=1, zp_in=zp_in,
                  zp_out=-5, act=act)
    x = r.integers(-128, 128, B * H * W * C).astype(np.int8)
    w = r.integers(-127, 128, 9 * C).astype(np.int8)
    b, m, s = random_quant(r, C)
    got = run_op_model(ctx, d, B, x, w, b, m, s)
    _check(got, oracle_mod.op_s8(d, B, x, w, b, m, s))


@pytest.mark.parametrize("B,H,W,C,stride,pads,zp_in,act", [
    (2, 8, 256, 64, 2, None, -128, (-128, 127)),         # stride 2, SAME (bottom/right pad)
    (3, 9, 258, 64, 2, (1, 1, 1, 1), 5, (-20, 90)),      # stride 2, top/left pad, clamp
    (2, 6, 256, 128, 2, None, 0, (-128, 127)),           # two channel blocks, stride 2
    (2, 7, 128, 256, 1, None, -3, (0, 127)),             # four channel blocks, stride 1
    (1, 12, 200, 128, 1, None, 9, (-128, 127)),          # partial second tile, channel blocks
    (2, 1, 160, 64, 1, None, 2, (-128, 127)),            # one row, partial second tile
    (2, 2, 256, 32, 2, None, -7, (-128, 127)),           # one output row, stride 2
    (2, 6, 128, 128, 2, None, 0, (-128, 127)),           # stride 2, 64-px rows: two per tile
    (3, 5, 64, 256, 1, None, -128, (0, 127)),            # two per tile, odd batch
    (5, 4, 32, 128, 1, None, 4, (-128, 127)),            # 32-px rows: four per tile, partial group
    (2, 12, 64, 256, 2, None, -128, (-128, 127)),        # stride 2, 32-px rows: four per tile
    (3, 8, 96, 128, 2, None, 7, (-30, 100)),             # stride 2, 48-px rows, partial group
    (5, 6, 48, 64, 2, None, -128, (0, 127)),             # stride 2, 24-px rows, partial group
    (3, 7, 50, 64, 1, None, 3, (-30, 100)),              # 50-px rows, clamp
    (2, 9, 40, 64, 2, (1, 1, 1, 1), -2, (-128, 127)),    # stride 2 top/left pad, narrow
    (6, 6, 32, 512, 1, None, -128, (-128, 127)),         # eight channel blocks, four per tile
    (3, 6, 24, 512, 1, None, 3, (-20, 110)),             # eight blocks, 24-px rows, clamp
])
def test_depthwise_row_streaming_shapes(ctx, oracle_mod, B, H, W, C, stride, pads, zp_in, act):
    """Depthwise shapes of the row-streaming tensor-core kernel beyond the
    config-3 blocks: stride 2 (even/odd pixel boxes), channel blocks (one
    block per CTA), partial column tiles, and stride-1 rows of at most 64
    or 32 pixels with two or four samples packed into one 128-row tile
    (narrow stride-2 rows run on the CUDA-core kernel)."""
    r = np.random.default_rng(7300 + H * W + C + stride)
    if pads is None:
        d = conv_desc(capi.OP_DEPTHWISE_CONV2D, H, W, C, C, k=3, stride=stride, zp_in=zp_in,
                      zp_out=-6, act=act)
    else:
        pt, pb, pl, pr = pads
        ho = (H + pt + pb - 3) // stride + 1
        wo = (W + pl + pr - 3) // stride + 1
        d = make_desc(kind=capi.OP_DEPTHWISE_CONV2D, in_h=H, in_w=W, in_c=C, out_h=ho, out_w=wo,
                      out_c=C, kernel_h=3, kernel_w=3, stride_h=stride, stride_w=stride,
                      pad_top=pt, pad_left=pl, pad_bottom=pb, pad_right=pr, zp_in=zp_in,
                      zp_out=-6, act_min=act[0], act_max=act[1])
    x = r.integers(-128, 128, B * H * W * C).astype(np.int8)
    w = r.integers(-127, 128, 9 * C).astype(np.int8)
    b, m, s = random_quant(r, C)
    got = run_op_model(ctx, d, B, x, w, b, m, s)
    _check(got, oracle_mod.op_s8(d, B, x, w, b, m, s))


@pytest.mark.parametrize("B,H,W,K,N,act", [
    (2, 8, 64, 32, 64, (-128, 127)),     # 256-row tiles
    (3, 5, 33, 64, 32, (-10, 100)),      # 256-row tiles, ragged last tile, clamp
    (2, 6, 40, 128, 128, (-128, 127)),
    (1, 4, 50, 64, 256, (0, 127)),
    # Several 128-column N tiles (run-time table offsets, one N tile per CTA)
    (2, 6, 32, 256, 512, (-128, 127)),
    (3, 5, 21, 512, 384, (-20, 90)),     # ragged last row tile, clamp
    (1, 3, 7, 128, 320, (-128, 127)),    # last N tile partial
    (2, 5, 30, 64, 200, (-128, 127)),    # one 256-column tile, its second half partial
])
def test_pointwise_static_table(ctx, oracle_mod, B, H, W, K, N, act):
    r = np.random.default_rng(8000 + H * W + K + N)
    d = make_desc(kind=capi.OP_CONV2D, in_h=H, in_w=W, in_c=K, out_h=H, out_w=W, out_c=N,
                  zp_in=-128, zp_out=3, act_min=act[0], act_max=act[1])
    x = r.integers(-128, 128, B * H * W * K).astype(np.int8)
    w = r.integers(-127, 128, N * K).astype(np.int8)
    b, m, s = random_quant(r, N)
    got = run_op_model(ctx, d, B, x, w, b, m, s)
    _check(got, oracle_mod.op_s8(d, B, x, w, b, m, s))


@pytest.mark.parametrize("B,H,W,C,N,dw_act,pw_act", [
    (2, 4, 256, 32, 64, (-128, 127), (-128, 127)),   # config-3 block 0
    (2, 3, 256, 64, 64, (-128, 127), (-128, 127)),   # block 1
    (2, 2, 200, 64, 64, (-100, 120), (-20, 90)),      # partial tile, both clamps
    (1, 5, 130, 32, 64, (0, 127), (-128, 127)),
    (2, 7, 300, 32, 64, (4, 127), (-128, 127)),       # 32 channels: floor form, 3 column tiles
    (3, 9, 128, 32, 64, (-128, 127), (-30, 60)),      # 32 channels: pointwise clamp
    (3, 3, 128, 128, 128, (-128, 127), (-128, 127)),  # not fused: two kernels
])
def test_depthwise_pointwise_pair(ctx, oracle_mod, B, H, W, C, N, dw_act, pw_act):
    """A depthwise conv followed by a 1x1 conv: the compiled model runs the
    pair as one kernel where the shapes allow (the depthwise output stays in
    shared memory); the pointwise output must equal the oracle's two ops in
    sequence."""
    r = np.random.default_rng(9000 + H * W + C + N)
    dw = conv_desc(capi.OP_DEPTHWISE_CONV2D, H, W, C, C, k=3, stride=1, zp_in=-7, zp_out=4,
                   act=dw_act)
    pw = make_desc(kind=capi.OP_CONV2D, in_h=H, in_w=W, in_c=C, out_h=H, out_w=W, out_c=N,
                   zp_in=4, zp_out=-2, act_min=pw_act[0], act_max=pw_act[1])
    x = r.integers(-128, 128, B * H * W * C).astype(np.int8)
    wd = r.integers(-127, 128, 9 * C).astype(np.int8)
    bd, md, sd = random_quant(r, C)
    wp = r.integers(-127, 128, N * C).astype(np.int8)
    bp, mp, sp = random_quant(r, N)
    got = run_chain_model(ctx, [(dw, wd, bd, md, sd), (pw, wp, bp, mp, sp)], B, x)
    mid = oracle_mod.op_s8(dw, B, x, wd, bd, md, sd)
    _check(got, oracle_mod.op_s8(pw, B, mid, wp, bp, mp, sp))


@pytest.mark.parametrize("B,H,W,stride,zp_in,act", [
    (2, 96, 512, 2, 0, (-128, 127)),     # the config-3 stem
    (3, 17, 33, 2, -5, (-20, 100)),      # odd sizes, clamp
    (2, 9, 10, 1, 3, (0, 127)),
])
def test_stem_conv_static_table(ctx, oracle_mod, B, H, W, stride, zp_in, act):
    """3x3 conv with one input and 32 output channels: the compiled model
    runs it with the weights and requant constants as kernel-parameter
    operands."""
    r = np.random.default_rng(7700 + H * W + stride)
    d = conv_desc(capi.OP_CONV2D, H, W, 1, 32, k=3, stride=stride, zp_in=zp_in, zp_out=-128,
                  act=act)
    x = r.integers(-128, 128, B * H * W).astype(np.int8)
    w = r.integers(-127, 128, 32 * 9).astype(np.int8)
    b, m, s = random_quant(r, 32)
    got = run_op_model(ctx, d, B, x, w, b, m, s)
    _check(got, oracle_mod.op_s8(d, B, x, w, b, m, s))


def _dw(H, W, C, stride, zp_in, zp_out, act):
    return conv_desc(capi.OP_DEPTHWISE_CONV2D, H, W, C, C, k=3, stride=stride, zp_in=zp_in,
                     zp_out=zp_out, act=act)


def _pw(H, W, K, N, zp_in, zp_out, act):
    return make_desc(kind=capi.OP_CONV2D, in_h=H, in_w=W, in_c=K, out_h=H, out_w=W, out_c=N,
                     zp_in=zp_in, zp_out=zp_out, act_min=act[0], act_max=act[1])


def _fc(K, N, zp_in, zp_out, act):
    return make_desc(kind=capi.OP_FULLY_CONNECTED, in_h=1, in_w=1, in_c=K, out_h=1, out_w=1,
                     out_c=N, zp_in=zp_in, zp_out=zp_out, act_min=act[0], act_max=act[1])


# Ops whose clamp starts at or above the output zero point (ReLU and the
# like) take the floor form of the requantisation in every kernel: the
# negative-accumulator rounding term is left out (those outputs clamp to
# act_min either way) and the table holds the bias folded into the 64-bit
# addend.  Each case: (label, batch, op descs of a chain).
FLOOR_CASES = [
    ("dw_tc static, clamp", 1, [_dw(6, 384, 96, 1, -3, -5, (-5, 127))]),
    ("dw_tc static, zp -128", 2, [_dw(4, 200, 96, 1, 7, -128, (-128, 127))]),
    ("row-streaming s1", 2, [_dw(5, 256, 64, 1, 3, -128, (-128, 127))]),
    ("row-streaming s2 blocks, clamp", 2, [_dw(8, 256, 128, 2, -128, 10, (10, 127))]),
    ("row-streaming packed rows", 3, [_dw(5, 32, 256, 1, -128, -128, (-128, 127))]),
    ("row-streaming 512 channels", 5, [_dw(6, 32, 512, 1, 2, -128, (-128, 127))]),
    ("cuda-core dw s2, clamp", 2, [_dw(6, 128, 128, 2, 0, -6, (-6, 127))]),
    ("cuda-core dw s1, 36 channels", 2, [_dw(5, 40, 36, 1, 2, -128, (-128, 120))]),
    ("gemm static 128", 2, [_pw(6, 40, 64, 128, -128, -128, (-128, 127))]),
    ("gemm static 256-row tiles, clamp", 2, [_pw(8, 64, 32, 64, 5, 3, (3, 100))]),
    ("gemm static 256 columns", 2, [_pw(6, 40, 64, 256, -128, -128, (-128, 127))]),
    ("gemm static 256 columns, clamp", 3, [_pw(5, 33, 128, 256, 2, 3, (3, 90))]),
    ("gemm 200 columns, run-time offsets", 2, [_pw(4, 30, 64, 200, -128, -128, (-128, 127))]),
    ("gemm 512 columns, run-time offsets", 2, [_pw(6, 32, 256, 512, -128, -128, (-128, 127))]),
    ("gemm 384 columns, run-time offsets, clamp", 3, [_pw(5, 21, 128, 384, 3, 4, (4, 110))]),
    ("gemm 3x3 table", 2, [conv_desc(capi.OP_CONV2D, 9, 20, 32, 64, k=3, stride=1, zp_in=-128,
                                     zp_out=-128, act=(-128, 127))]),
    ("gemm 3x3 table, clamp", 2, [conv_desc(capi.OP_CONV2D, 7, 12, 16, 48, k=3, stride=1,
                                            zp_in=4, zp_out=5, act=(5, 127))]),
    ("fc", 300, [_fc(256, 100, -3, -128, (-128, 127))]),
    ("stem table", 2, [conv_desc(capi.OP_CONV2D, 20, 64, 1, 32, k=3, stride=2, zp_in=0,
                                 zp_out=-100, act=(-100, 127))]),
    ("small conv in_c 3", 2, [conv_desc(capi.OP_CONV2D, 16, 16, 3, 32, k=3, stride=1,
                                        zp_in=-128, zp_out=-128, act=(-128, 127))]),
    ("dw+pw pair 32->64", 2, [_dw(4, 256, 32, 1, -7, -128, (-128, 127)),
                              _pw(4, 256, 32, 64, -128, 2, (2, 127))]),
    ("dw+pw pair 64->64 (row-streaming)", 2, [_dw(3, 256, 64, 1, 5, 6, (6, 127)),
                                              _pw(3, 256, 64, 64, 6, -128, (-128, 127))]),
    ("dw+pw pair, pointwise not floor", 2, [_dw(3, 256, 64, 1, 5, -128, (-128, 127)),
                                            _pw(3, 256, 64, 64, -128, 0, (-128, 127))]),
]


def _weights(r, d):
    kind = int(d["kind"])
    if kind == capi.OP_DEPTHWISE_CONV2D:
        n = 9 * int(d["in_c"])
    elif kind == capi.OP_FULLY_CONNECTED:
        n = int(d["in_c"]) * int(d["out_c"])
    else:
        n = int(d["out_c"]) * int(d["kernel_h"]) * int(d["kernel_w"]) * int(d["in_c"])
    return r.integers(-127, 128, n).astype(np.int8)


@pytest.mark.parametrize("label,B,descs", FLOOR_CASES, ids=[c[0] for c in FLOOR_CASES])
def test_floor_form_paths(ctx, oracle_mod, label, B, descs):
    r = np.random.default_rng(zlib.crc32(label.encode()))
    ops = []
    for d in descs:
        b, m, s = random_quant(r, int(d["out_c"]))
        ops.append((d, _weights(r, d), b, m, s))
    d0 = descs[0]
    x = r.integers(-128, 128, B * int(d0["in_h"]) * int(d0["in_w"]) * int(d0["in_c"]))
    x = x.astype(np.int8)
    got = run_chain_model(ctx, ops, B, x)
    want = x
    for d, w, b, m, s in ops:
        want = oracle_mod.op_s8(d, B, want, w, b, m, s)
    _check(got, want)


@pytest.mark.parametrize("B,H,W,pads,zp_in,zp_out,act", [
    (2, 96, 512, None, 0, -128, (-128, 127)),      # the config-3 stem (floor form)
    (2, 20, 72, None, -9, 10, (-128, 127)),        # fast form, 36 px rows (partial warp)
    (3, 11, 64, (1, 1, 0, 1), 5, 10, (-50, 100)),  # top padding, clamp, fast form
    (2, 14, 256, (2, 0, 0, 1), -128, 7, (7, 90)),  # two rows of top padding, floor + clamp
    (1, 7, 16, (0, 0, 0, 0), 3, -128, (-128, 127)),  # VALID: last input column unused
])
def test_stem_stride2_register_kernel(ctx, oracle_mod, B, H, W, pads, zp_in, zp_out, act):
    """3x3 stride-2 conv with one input and 32 output channels on rows of a
    multiple of 8 bytes: the register-resident stem kernel (four pixels x
    eight channels per thread, strips of output rows)."""
    r = np.random.default_rng(7800 + H * W + zp_out)
    if pads is None:
        d = conv_desc(capi.OP_CONV2D, H, W, 1, 32, k=3, stride=2, zp_in=zp_in, zp_out=zp_out,
                      act=act)
    else:
        pt, pb, pl, pr = pads
        d = make_desc(kind=capi.OP_CONV2D, in_h=H, in_w=W, in_c=1,
                      out_h=(H + pt + pb - 3) // 2 + 1, out_w=(W + pl + pr - 3) // 2 + 1,
                      out_c=32, kernel_h=3, kernel_w=3, stride_h=2, stride_w=2, pad_top=pt,
                      pad_left=pl, pad_bottom=pb, pad_right=pr, zp_in=zp_in, zp_out=zp_out,
                      act_min=act[0], act_max=act[1])
    x = r.integers(-128, 128, B * H * W).astype(np.int8)
    w = r.integers(-127, 128, 32 * 9).astype(np.int8)
    b, m, s = random_quant(r, 32)
    got = run_op_model(ctx, d, B, x, w, b, m, s)
    _check(got, oracle_mod.op_s8(d, B, x, w, b, m, s))
