"""ctypes binding of the CPU oracle (oracle/_build/liboracle.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, the smoke check and the
benchmark's CPU-baseline leg as the checker; the product never imports it.
"""
from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "_build" / "liboracle.so"

_lib = None
_i64p = ctypes.POINTER(ctypes.c_int64)
_fp = ctypes.POINTER(ctypes.c_float)
_vp = ctypes.c_void_p


def build() -> None:
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        l = ctypes.CDLL(str(LIB_PATH))
        for name in ("orc_f32_conv2d", "orc_f32_conv2d_relu"):
            getattr(l, name).argtypes = [_fp, _i64p, _fp, _i64p, _fp, _i64p, _i64p, _fp, _i64p]
        l.orc_f32_max_pool2d.argtypes = [_fp, _i64p, _i64p, _i64p, _fp, _i64p]
        l.orc_f32_reshape.argtypes = [_fp, _fp, ctypes.c_int64]
        for name in ("orc_f32_fully_connected", "orc_f32_fully_connected_relu"):
            getattr(l, name).argtypes = [_fp, ctypes.c_int64, _fp, _fp, _fp, ctypes.c_int64]
        l.orc_f32_matmul_bt.argtypes = [_fp, _fp, _fp, ctypes.c_int64, ctypes.c_int64,
                                        ctypes.c_int64]
        l.orc_f32_matmul_bt_tiled.argtypes = [_fp, _fp, _fp, ctypes.c_int64, ctypes.c_int64,
                                              ctypes.c_int64]
        l.orc_f32_relu.argtypes = [_fp, ctypes.c_int64]
        l.orc_f32_im2col.argtypes = [_fp, _i64p, _i64p, _i64p, _i64p, _i64p, _fp]
        l.orc_f32_im2col_padded.argtypes = [_fp, _i64p, _i64p, _i64p, _i64p, _fp]
        l.orc_f32_bias_add.argtypes = [_fp, _fp, ctypes.c_int64, ctypes.c_int64]
        l.orc_same_padding.argtypes = [ctypes.c_int64] * 6 + [_i64p]
        l.orc_srdhm.argtypes = [ctypes.c_int32, ctypes.c_int32]
        l.orc_srdhm.restype = ctypes.c_int32
        l.orc_rdbpot.argtypes = [ctypes.c_int32, ctypes.c_int32]
        l.orc_rdbpot.restype = ctypes.c_int32
        l.orc_mbqm.argtypes = [ctypes.c_int32, ctypes.c_int32, ctypes.c_int32]
        l.orc_mbqm.restype = ctypes.c_int32
        l.orc_quantize_multiplier.argtypes = [ctypes.c_double, ctypes.POINTER(ctypes.c_int32),
                                              ctypes.POINTER(ctypes.c_int32)]
        l.orc_op_s8.argtypes = [_vp, ctypes.c_int64, _vp, _vp, _vp, _vp, _vp, _vp]
        l.orc_op_s8.restype = ctypes.c_int
        l.orc_net_forward_s8.argtypes = [_vp, ctypes.c_int32, _vp, ctypes.c_int64, _vp, _vp,
                                         ctypes.c_int32]
        l.orc_net_forward_s8.restype = ctypes.c_int
        _lib = l
    return _lib


def _f(a: np.ndarray):
    assert a.dtype == np.float32 and a.flags.c_contiguous
    return a.ctypes.data_as(_fp)


def _shape(v) -> ctypes.Array:
    return (ctypes.c_int64 * len(v))(*[int(x) for x in v])


# ------------------------------------------------------------------- f32
def f32_conv2d(x, in_shape, w, w_shape, bias, stride, padding, out_shape, relu=False):
    out = np.zeros(int(np.prod(out_shape)), dtype=np.float32)
    fn = lib().orc_f32_conv2d_relu if relu else lib().orc_f32_conv2d
    fn(_f(x), _shape(in_shape), _f(w), _shape(w_shape),
       _f(bias) if bias is not None else None, _shape(stride), _shape(padding), _f(out),
       _shape(out_shape))
    return out


def f32_max_pool2d(x, in_shape, kernel, stride, out_shape):
    out = np.zeros(int(np.prod(out_shape)), dtype=np.float32)
    lib().orc_f32_max_pool2d(_f(x), _shape(in_shape), _shape(kernel), _shape(stride), _f(out),
                             _shape(out_shape))
    return out


def f32_fully_connected(x, in_f, w, b, out_f, relu=False):
    out = np.zeros(out_f, dtype=np.float32)
    fn = lib().orc_f32_fully_connected_relu if relu else lib().orc_f32_fully_connected
    fn(_f(x), in_f, _f(w), _f(b), _f(out), out_f)
    return out


def f32_matmul_bt(a, b, m, k, n):
    c = np.zeros(m * n, dtype=np.float32)
    lib().orc_f32_matmul_bt(_f(a), _f(b), _f(c), m, k, n)
    return c


def f32_matmul_bt_tiled(a, b, mt, kt, nt):
    c = np.zeros(mt * 4 * nt * 4, dtype=np.float32)
    lib().orc_f32_matmul_bt_tiled(_f(a), _f(b), _f(c), mt, kt, nt)
    return c


def f32_relu(x):
    y = np.array(x, dtype=np.float32, copy=True)
    lib().orc_f32_relu(_f(y), y.size)
    return y


def f32_bias_add(x, bias, rows, cols):
    y = np.array(x, dtype=np.float32, copy=True)
    lib().orc_f32_bias_add(_f(y), _f(np.ascontiguousarray(bias, dtype=np.float32)), rows, cols)
    return y


def f32_im2col(x, in_shape, kernel, stride, padding, out_hw):
    n = in_shape[0] * out_hw[0] * out_hw[1] * kernel[0] * kernel[1] * in_shape[3]
    col = np.zeros(n, dtype=np.float32)
    lib().orc_f32_im2col(_f(x), _shape(in_shape), _shape(kernel), _shape(stride),
                         _shape(padding), _shape(out_hw), _f(col))
    return col


def f32_im2col_padded(x, in_shape, kernel, padding, out_hw, fill=0.0):
    k = kernel[0] * kernel[1] * in_shape[3]
    kp = (k + 3) // 4 * 4
    col = np.full(in_shape[0] * out_hw[0] * out_hw[1] * kp, fill, dtype=np.float32)
    lib().orc_f32_im2col_padded(_f(x), _shape(in_shape), _shape(kernel), _shape(padding),
                                _shape(out_hw), _f(col))
    return col


def same_padding(in_h, in_w, k_h, k_w, s_h, s_w):
    out = (ctypes.c_int64 * 4)()
    lib().orc_same_padding(in_h, in_w, k_h, k_w, s_h, s_w, out)
    return tuple(out)


# ------------------------------------------------------------------ int8
def srdhm(a: int, b: int) -> int:
    return lib().orc_srdhm(a, b)


def rdbpot(x: int, e: int) -> int:
    return lib().orc_rdbpot(x, e)


def mbqm(x: int, m: int, s: int) -> int:
    return lib().orc_mbqm(x, m, s)


def quantize_multiplier(real: float) -> tuple[int, int]:
    m, s = ctypes.c_int32(), ctypes.c_int32()
    lib().orc_quantize_multiplier(real, ctypes.byref(m), ctypes.byref(s))
    return m.value, s.value


def op_s8(desc, batch, x, filt=None, bias=None, mult=None, shift=None):
    """One int8 op over `batch` samples; desc is a record of pspml_op_desc."""
    d = np.ascontiguousarray(np.array(desc).reshape(1))
    out_elems = int(d["out_h"][0]) * int(d["out_w"][0]) * int(d["out_c"][0])
    out = np.zeros(batch * out_elems, dtype=np.int8)
    x = np.ascontiguousarray(x, dtype=np.int8)

    def p(a, dt):
        return None if a is None else np.ascontiguousarray(a, dtype=dt).ctypes.data

    keep = [np.ascontiguousarray(a) for a in (filt, bias, mult, shift) if a is not None]
    rc = lib().orc_op_s8(d.ctypes.data, batch, x.ctypes.data, p(filt, np.int8),
                         p(bias, np.int32), p(mult, np.int32), p(shift, np.int32),
                         out.ctypes.data)
    del keep
    if rc != 0:
        raise RuntimeError("oracle op failed")
    return out


def net_forward_s8(descs: np.ndarray, blob: np.ndarray, x: np.ndarray, threads: int = 0):
    descs = np.ascontiguousarray(descs)
    blob = np.ascontiguousarray(blob, dtype=np.uint8)
    x = np.ascontiguousarray(x, dtype=np.int8)
    batch = x.shape[0]
    last = descs[-1]
    out = np.zeros((batch, int(last["out_h"]) * int(last["out_w"]) * int(last["out_c"])),
                   dtype=np.int8)
    rc = lib().orc_net_forward_s8(descs.ctypes.data, len(descs), blob.ctypes.data, batch,
                                  x.ctypes.data, out.ctypes.data, threads)
    if rc != 0:
        raise RuntimeError("oracle network forward failed")
    return out
