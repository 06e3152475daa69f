"""3x3 convs with 2, 3, 4 or 8 input channels on the tensor cores
(csrc/im2col_tc.cu), bit-exact against the oracle.

A compiled model runs such a conv (32 or 64 outputs, every channel in the
fast requantisation form) as patches gathered into a shared-memory A tile
and one to three tcgen05 MMAs per 128 output pixels; each thread of the
epilogue requantises a fixed set of channels of four pixels (16x256b
tensor-memory loads) and lanes exchange channel pairs before the store.
Cases cover the config-2 first conv (3 -> 32, 64 x 64), tiles of several rows
(rows of 28 and 14 pixels, the last tile of a sample partial), rows wider
than 128 pixels (several tiles per row, a partial last one), stride 2 with
odd sizes, valid padding, rows copied in 4-byte units (row bytes not a
multiple of 16), the four requantisation forms (floor / fast, with and
without a clamp narrower than int8) and input zero points that make the
padding matter.
"""
import numpy as np
import pytest

from gpu_helpers import conv_desc, random_quant
from pspml import capi

pytestmark = pytest.mark.gpu

# (zp_out, act): ep_flags 2 (floor), 0 (fast), 3 (floor + clamp), 1 (fast + clamp)
FORMS = {
    "floor": (-128, (-128, 127)),
    "fast": (0, (-128, 127)),
    "floor_clamp": (-128, (-128, 100)),
    "fast_clamp": (5, (-100, 120)),
}


def _single_conv(H, W, ci, co, stride, pad, zp_in, form, seed):
    r = np.random.default_rng(seed)
    zp_out, act = FORMS[form]
    d = conv_desc(capi.OP_CONV2D, H, W, ci, co, k=3, stride=stride, pad=pad, zp_in=zp_in,
                  zp_out=zp_out, act=act)
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
    descs = np.array(d).reshape(1)
    descs["filter_off"][0], descs["bias_off"][0], descs["mult_off"][0], descs["shift_off"][0] = offs
    return descs, blob


def _run(ctx, oracle_mod, descs, blob, batch, micro, seed):
    import torch
    r = np.random.default_rng(seed)
    H, W, ci = int(descs[0]["in_h"]), int(descs[0]["in_w"]), int(descs[0]["in_c"])
    x = r.integers(-128, 128, (batch, H, W, ci)).astype(np.int8)
    model = capi.Model(ctx, descs, blob, micro)
    xi = torch.from_numpy(x.reshape(-1)).cuda()
    out = torch.full((batch * model.out_bytes,), 77, dtype=torch.int8, device="cuda")
    model.forward_device(xi.data_ptr(), out.data_ptr(), batch,
                         torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    ctx.check_device()
    model.close()
    got = out.cpu().numpy().reshape(batch, -1)
    want = oracle_mod.net_forward_s8(descs, blob, x)
    return got, want


def _check(got, want):
    mism = np.flatnonzero(got != want)
    assert mism.size == 0, (f"{mism.size} of {want.size} differ; first at {mism[:5]}: "
                            f"got {got.reshape(-1)[mism[:5]]} want {want.reshape(-1)[mism[:5]]}")


@pytest.mark.parametrize("H,W,ci,co,stride,pad,zp_in,form,batch", [
    (64, 64, 3, 32, 1, "same", -3, "floor", 5),        # config-2 first conv
    (28, 28, 2, 32, 1, "same", -128, "fast", 4),       # four 28-px rows per tile
    (14, 14, 8, 32, 1, "same", 11, "floor_clamp", 6),  # nine rows per tile
    (9, 12, 2, 64, 1, "same", 40, "fast_clamp", 5),
    (13, 200, 4, 64, 1, "same", -7, "fast", 2),        # 2 tiles per row, the last partial
    (17, 20, 4, 64, 2, "same", 25, "floor", 3),
    (31, 132, 3, 64, 2, "same", -60, "fast_clamp", 2),
    (12, 300, 2, 32, 2, "valid", 0, "fast", 2),        # 600-byte rows: 4-byte copies
    (10, 36, 8, 32, 1, "valid", -128, "floor_clamp", 3),
    (1, 8, 2, 32, 1, "same", 90, "floor", 7),          # one row
    (5, 4, 3, 32, 2, "same", -1, "fast", 9),           # odd sizes, stride 2
    (96, 512, 2, 32, 2, "same", -128, "floor", 2),     # wide stride-2 rows
])
def test_im2col_conv(ctx, oracle_mod, H, W, ci, co, stride, pad, zp_in, form, batch):
    seed = 7 * H + W + 13 * ci + co + stride + zp_in + 1000
    descs, blob = _single_conv(H, W, ci, co, stride, pad, zp_in, form, seed)
    got, want = _run(ctx, oracle_mod, descs, blob, batch, batch, seed + 1)
    _check(got, want)


def test_im2col_conv_micro_batches(ctx, oracle_mod):
    """Several micro-batches, the last ragged, through one model."""
    descs, blob = _single_conv(64, 64, 3, 32, 1, "same", -128, "floor", 4242)
    got, want = _run(ctx, oracle_mod, descs, blob, 11, 4, 4243)
    _check(got, want)
