"""Helpers shared by the GPU parity tests: op descriptors, random quantised
layers, and running one op through the C ABI on torch-owned device memory."""
from __future__ import annotations

import ctypes
import math

import numpy as np

from pspml import capi, netspec


def make_desc(**kw) -> np.void:
    d = np.zeros(1, dtype=capi.OP_DESC_DTYPE)[0]
    base = dict(kernel_h=1, kernel_w=1, stride_h=1, stride_w=1, act_min=-128, act_max=127,
                filter_off=-1, bias_off=-1, mult_off=-1, shift_off=-1)
    base.update(kw)
    for k, v in base.items():
        d[k] = v
    return d


def conv_desc(kind, n_h, n_w, ci, co, k=3, stride=1, pad="same", zp_in=-128, zp_out=0,
              act=(-128, 127)):
    if pad == "same":
        pt, pb, pl, pr = netspec.same_padding(n_h, n_w, k, k, stride, stride)
    else:
        pt = pb = pl = pr = 0
    ho = (n_h + pt + pb - k) // stride + 1
    wo = (n_w + pl + pr - k) // stride + 1
    return make_desc(kind=kind, in_h=n_h, in_w=n_w, in_c=ci, out_h=ho, out_w=wo, out_c=co,
                     kernel_h=k, kernel_w=k, stride_h=stride, stride_w=stride, pad_top=pt,
                     pad_left=pl, pad_bottom=pb, pad_right=pr, zp_in=zp_in, zp_out=zp_out,
                     act_min=act[0], act_max=act[1])


def random_quant(rng, n, mode="calibrated"):
    """Per-channel (bias, mult, shift).  `extreme` mixes edge multipliers:
    exactly 2**30, 2**31 - 1, left shifts and the 31-bit right shift."""
    bias = rng.integers(-4096, 4097, n).astype(np.int32)
    mult = np.zeros(n, np.int32)
    shift = np.zeros(n, np.int32)
    for c in range(n):
        real = math.exp(rng.uniform(math.log(1e-5), math.log(2e-2)))
        mult[c], shift[c] = netspec.quantize_multiplier(real)
    if mode == "extreme":
        bias = rng.integers(-(1 << 20), 1 << 20, n).astype(np.int32)
        choices = [(1 << 30, 0), ((1 << 31) - 1, -1), (1 << 30, 1), ((3 << 29), -31),
                   (1 << 30, -12), (1234567890, 2), ((1 << 31) - 1, -20)]
        for c in range(n):
            mult[c], shift[c] = choices[c % len(choices)]
    return bias, mult, shift


def out_elems(d) -> int:
    return int(d["out_h"]) * int(d["out_w"]) * int(d["out_c"])


def in_elems(d) -> int:
    return int(d["in_h"]) * int(d["in_w"]) * int(d["in_c"])


_FN = {
    capi.OP_CONV2D: "pspml_conv2d_s8",
    capi.OP_DEPTHWISE_CONV2D: "pspml_depthwise_conv2d_s8",
    capi.OP_FULLY_CONNECTED: "pspml_fully_connected_s8",
    capi.OP_MAX_POOL2D: "pspml_max_pool2d_s8",
    capi.OP_AVERAGE_POOL2D: "pspml_average_pool2d_s8",
}


def run_op_gpu(ctx, d, batch, x, filt=None, bias=None, mult=None, shift=None):
    """Runs one op through the C ABI; returns the int8 output (host)."""
    import torch

    def dev(a, dt):
        if a is None:
            return None, None
        t = torch.from_numpy(np.ascontiguousarray(a, dtype=dt)).cuda()
        return t, ctypes.c_void_p(t.data_ptr())

    xt, xp = dev(x.reshape(-1), np.int8)
    _, fp = dev(filt, np.int8)
    bt, bp = dev(bias, np.int32)
    mt, mp = dev(mult, np.int32)
    st, sp = dev(shift, np.int32)
    out = torch.full((max(1, batch * out_elems(d)),), 99, dtype=torch.int8, device="cuda")
    op = ctypes.c_void_p(out.data_ptr())
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    ds = capi.desc_struct(d)
    kind = int(d["kind"])
    fn = _FN[kind]
    if kind in (capi.OP_MAX_POOL2D, capi.OP_AVERAGE_POOL2D):
        capi.call(fn, ctx.handle, ctypes.byref(ds), batch, xp, op, stream)
    else:
        capi.call(fn, ctx.handle, ctypes.byref(ds), batch, xp, fp, bp, mp, sp, op, stream)
    torch.cuda.synchronize()
    ctx.check_device()
    return out.cpu().numpy()[: batch * out_elems(d)]


def run_op_model(ctx, d, batch, x, filt, bias, mult, shift, micro=None):
    """Runs one weighted op as a one-op compiled model (weights uploaded with
    the model; the host builds the constant requant table when every
    channel takes the fast form, so this exercises the constant-table
    kernels); returns the int8 output (host)."""
    return run_chain_model(ctx, [(d, filt, bias, mult, shift)], batch, x, micro)


def run_chain_model(ctx, ops, batch, x, micro=None):
    """Runs a chain of weighted ops [(desc, filter, bias, mult, shift)] as
    one compiled model; returns the last op's int8 output (host)."""
    import torch

    parts, descs = [], []
    for d, filt, bias, mult, shift in ops:
        parts += [np.ascontiguousarray(filt, np.int8).view(np.uint8).reshape(-1),
                  np.ascontiguousarray(bias, np.int32).view(np.uint8).reshape(-1),
                  np.ascontiguousarray(mult, np.int32).view(np.uint8).reshape(-1),
                  np.ascontiguousarray(shift, np.int32).view(np.uint8).reshape(-1)]
        descs.append(np.array(d).reshape(1).copy())
    offs, pos = [], 0
    for a in parts:
        offs.append(pos)
        pos += (a.size + 255) // 256 * 256
    blob = np.zeros(pos, np.uint8)
    for o, a in zip(offs, parts):
        blob[o:o + a.size] = a
    dd = np.concatenate(descs)
    for i in range(len(ops)):
        (dd["filter_off"][i], dd["bias_off"][i], dd["mult_off"][i],
         dd["shift_off"][i]) = offs[4 * i:4 * i + 4]
    model = capi.Model(ctx, dd, blob, micro or batch)
    xi = torch.from_numpy(np.ascontiguousarray(x, np.int8).reshape(-1)).cuda()
    out = torch.full((batch * out_elems(ops[-1][0]),), 99, dtype=torch.int8, device="cuda")
    model.forward_device(xi.data_ptr(), out.data_ptr(), batch,
                         torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    ctx.check_device()
    model.close()
    return out.cpu().numpy()
