"""ctypes binding of libpspml_cuda.so (the C ABI declared in include/pspml.h).

The library is built in-tree by ``make -C psp-ml_b200``.  Loading fails
loudly when it is missing: there is no CPU fallback for any entry point.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

import numpy as np

LIB_PATH = Path(__file__).resolve().parent / "libpspml_cuda.so"

# pspml_status
OK = 0
ERR_INVALID_ARG = 1
ERR_UNSUPPORTED = 2
ERR_CUDA = 3
ERR_OOM = 4
ERR_TIMEOUT = 5
ERR_NO_DEVICE = 6
ERR_DEVICE_WAIT = 7
STATUS_NAMES = {
    OK: "OK", ERR_INVALID_ARG: "INVALID_ARG", ERR_UNSUPPORTED: "UNSUPPORTED",
    ERR_CUDA: "CUDA", ERR_OOM: "OOM", ERR_TIMEOUT: "TIMEOUT",
    ERR_NO_DEVICE: "NO_DEVICE", ERR_DEVICE_WAIT: "DEVICE_WAIT",
}

# pspml_op_kind (mirrors the TFLite builtins the reference lowers,
# cargo-psp-ml/src/parse/tflite/lowering.rs:92-104, plus DW conv and avg pool)
OP_CONV2D = 1
OP_DEPTHWISE_CONV2D = 2
OP_FULLY_CONNECTED = 3
OP_MAX_POOL2D = 4
OP_AVERAGE_POOL2D = 5
OP_RESHAPE = 6

# pspml_op_desc.flags bits of the f32 ops
F32_RELU = 1
F32_GEMM_ORDER = 2

# Byte-for-byte layout of struct pspml_op_desc.
OP_DESC_FIELDS_I32 = (
    "kind", "in_h", "in_w", "in_c", "out_h", "out_w", "out_c",
    "kernel_h", "kernel_w", "stride_h", "stride_w",
    "pad_top", "pad_left", "pad_bottom", "pad_right",
    "zp_in", "zp_out", "act_min", "act_max", "flags",
)
OP_DESC_FIELDS_I64 = ("filter_off", "bias_off", "mult_off", "shift_off")
OP_DESC_DTYPE = np.dtype(
    [(n, "<i4") for n in OP_DESC_FIELDS_I32] + [(n, "<i8") for n in OP_DESC_FIELDS_I64])
assert OP_DESC_DTYPE.itemsize == 112


class OpDesc(ctypes.Structure):
    _fields_ = ([(n, ctypes.c_int32) for n in OP_DESC_FIELDS_I32] +
                [(n, ctypes.c_int64) for n in OP_DESC_FIELDS_I64])


assert ctypes.sizeof(OpDesc) == OP_DESC_DTYPE.itemsize


class Timing(ctypes.Structure):
    _fields_ = [("total_ms", ctypes.c_double), ("h2d_bytes", ctypes.c_double),
                ("d2h_bytes", ctypes.c_double), ("micro_batches", ctypes.c_int32),
                ("devices", ctypes.c_int32), ("rerun_shards", ctypes.c_int32)]


class PspmlError(RuntimeError):
    def __init__(self, status: int, fn: str, msg: str):
        super().__init__(f"{fn} failed: {STATUS_NAMES.get(status, status)}: {msg}")
        self.status = status


# Every exported symbol with its argument types; include/pspml.h declares
# exactly these.
_vp = ctypes.c_void_p
_i32 = ctypes.c_int32
_i64 = ctypes.c_int64
_sz = ctypes.c_size_t
_PROTOS = {
    "pspml_last_error": (ctypes.c_char_p, []),
    "pspml_abi_version": (_i32, []),
    "pspml_device_count": (ctypes.c_int, [ctypes.POINTER(ctypes.c_int)]),
    "pspml_ctx_create": (ctypes.c_int, [ctypes.c_int, _sz, ctypes.POINTER(_vp)]),
    "pspml_ctx_destroy": (ctypes.c_int, [_vp]),
    "pspml_ctx_set_timeout_ms": (ctypes.c_int, [_vp, _i64]),
    "pspml_ctx_check_device": (ctypes.c_int, [_vp]),
    "pspml_ctx_wait_selftest": (ctypes.c_int, [_vp, _i64, _i32]),
    "pspml_host_alloc": (ctypes.c_int, [_sz, ctypes.POINTER(_vp)]),
    "pspml_host_free": (ctypes.c_int, [_vp]),
    "pspml_conv2d_s8": (ctypes.c_int, [_vp, _vp, _i64, _vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    "pspml_depthwise_conv2d_s8": (ctypes.c_int,
                                  [_vp, _vp, _i64, _vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    "pspml_fully_connected_s8": (ctypes.c_int,
                                 [_vp, _vp, _i64, _vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    "pspml_fully_connected_s8_noalloc": (ctypes.c_int,
                                         [_vp, _i64, _vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    "pspml_noalloc_check_device": (ctypes.c_int, []),
    "pspml_max_pool2d_s8": (ctypes.c_int, [_vp, _vp, _i64, _vp, _vp, _vp]),
    "pspml_average_pool2d_s8": (ctypes.c_int, [_vp, _vp, _i64, _vp, _vp, _vp]),
    "pspml_conv2d_f32": (ctypes.c_int, [_vp, _vp, _i64, _vp, _vp, _vp, _vp, _vp]),
    "pspml_max_pool2d_f32": (ctypes.c_int, [_vp, _vp, _i64, _vp, _vp, _vp]),
    "pspml_fully_connected_f32": (ctypes.c_int, [_vp, _vp, _i64, _vp, _vp, _vp, _vp, _vp]),
    "pspml_model_create": (ctypes.c_int, [_vp, _vp, _i32, _vp, _sz, _i32, ctypes.POINTER(_vp)]),
    "pspml_model_destroy": (ctypes.c_int, [_vp]),
    "pspml_model_info": (ctypes.c_int, [_vp, ctypes.POINTER(_sz), ctypes.POINTER(_sz),
                                        ctypes.POINTER(_sz)]),
    "pspml_model_op_fused": (ctypes.c_int, [_vp, _i32, ctypes.POINTER(_i32)]),
    "pspml_model_fail_next": (ctypes.c_int, [_vp, _i32, _i32]),
    "pspml_forward_device": (ctypes.c_int, [_vp, _vp, _vp, _i64, _vp]),
    "pspml_forward": (ctypes.c_int, [_vp, _vp, _vp, _i64, ctypes.POINTER(Timing)]),
    "pspml_forward_sharded": (ctypes.c_int, [ctypes.POINTER(_vp), _i32, _vp, _vp, _i64,
                                             ctypes.POINTER(Timing)]),
    "pspml_forward_timed": (ctypes.c_int, [_vp, _vp, _vp, _i64, ctypes.POINTER(ctypes.c_float),
                                           _vp]),
}

_lib = None


def load(path: str | os.PathLike | None = None) -> ctypes.CDLL:
    """Loads the C-ABI library (once) and declares every prototype."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = Path(path) if path is not None else LIB_PATH
    if not p.exists():
        raise FileNotFoundError(
            f"{p} is missing: build it with `make -C psp-ml_b200` (there is no CPU fallback)")
    lib = ctypes.CDLL(str(p))
    for name, (res, args) in _PROTOS.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if path is None:
        _lib = lib
    return lib


def exported_symbols() -> list[str]:
    return sorted(_PROTOS)


def check(status: int, fn: str) -> None:
    if status != OK:
        msg = load().pspml_last_error().decode(errors="replace")
        raise PspmlError(status, fn, msg)


def call(fn: str, *args) -> None:
    check(getattr(load(), fn)(*args), fn)


def device_count() -> int:
    n = ctypes.c_int(0)
    call("pspml_device_count", ctypes.byref(n))
    return n.value


def desc_struct(row: np.void | dict) -> OpDesc:
    """An OpDesc from a numpy OP_DESC_DTYPE record or a dict of fields."""
    d = OpDesc()
    for n in OP_DESC_FIELDS_I32 + OP_DESC_FIELDS_I64:
        setattr(d, n, int(row[n]))
    return d


class Context:
    """One device context (pspml_ctx)."""

    def __init__(self, device: int = 0, workspace_bytes: int = 0):
        self.lib = load()
        self.handle = ctypes.c_void_p()
        call("pspml_ctx_create", device, workspace_bytes, ctypes.byref(self.handle))
        self.device = device

    def close(self) -> None:
        if self.handle:
            self.lib.pspml_ctx_destroy(self.handle)
            self.handle = ctypes.c_void_p()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def set_timeout_ms(self, ms: int) -> None:
        call("pspml_ctx_set_timeout_ms", self.handle, ms)

    def check_device(self) -> None:
        call("pspml_ctx_check_device", self.handle)

    def wait_selftest(self, limit_us: int, signal: bool) -> None:
        call("pspml_ctx_wait_selftest", self.handle, limit_us, 1 if signal else 0)


class Model:
    """A compiled op chain on one device (pspml_model)."""

    def __init__(self, ctx: Context, ops: np.ndarray, blob: np.ndarray, max_micro_batch: int):
        ops = np.ascontiguousarray(ops, dtype=OP_DESC_DTYPE)
        blob = np.ascontiguousarray(blob, dtype=np.uint8)
        self.ctx = ctx
        self.lib = ctx.lib
        self.handle = ctypes.c_void_p()
        self.n_ops = len(ops)
        call("pspml_model_create", ctx.handle, ops.ctypes.data, len(ops),
             blob.ctypes.data, blob.nbytes, max_micro_batch, ctypes.byref(self.handle))
        a, b, c = ctypes.c_size_t(), ctypes.c_size_t(), ctypes.c_size_t()
        call("pspml_model_info", self.handle, ctypes.byref(a), ctypes.byref(b), ctypes.byref(c))
        self.in_bytes, self.out_bytes, self.arena_bytes = a.value, b.value, c.value

    def close(self) -> None:
        if self.handle:
            self.lib.pspml_model_destroy(self.handle)
            self.handle = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def op_fused(self, op: int) -> int:
        """0: op runs on its own; 1: its kernel also computes op + 1; 2: op - 1's
        kernel computes it."""
        f = ctypes.c_int32()
        call("pspml_model_op_fused", self.handle, op, ctypes.byref(f))
        return f.value

    def fail_next(self, count: int, status: int) -> None:
        """Host-side failure injection: the next `count` forward calls
        return `status` without touching the GPU."""
        call("pspml_model_fail_next", self.handle, count, status)

    def forward_device(self, dev_in: int, dev_out: int, batch: int, stream: int = 0) -> None:
        call("pspml_forward_device", self.handle, dev_in, dev_out, batch, stream)

    def forward(self, host_in: int, host_out: int, batch: int) -> Timing:
        t = Timing()
        call("pspml_forward", self.handle, host_in, host_out, batch, ctypes.byref(t))
        return t

    def forward_timed(self, dev_in: int, dev_out: int, batch: int, stream: int = 0) -> list[float]:
        ms = (ctypes.c_float * self.n_ops)()
        call("pspml_forward_timed", self.handle, dev_in, dev_out, batch, ms, stream)
        return list(ms)


def forward_sharded(models: list[Model], host_in: int, host_out: int, batch: int) -> Timing:
    arr = (ctypes.c_void_p * len(models))(*[m.handle.value for m in models])
    t = Timing()
    call("pspml_forward_sharded", arr, len(models), host_in, host_out, batch, ctypes.byref(t))
    return t
