"""The C-ABI library loads without a GPU and exports every function that
include/pspml.h declares (no compute calls)."""
import ctypes
import re
import subprocess
from pathlib import Path

import pytest

from pspml import capi

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "pspml.h"


def header_functions(path=HEADER):
    text = path.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(pspml_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    if not capi.LIB_PATH.exists():
        subprocess.run(["make", "-s", "-C", str(ROOT / "psp-ml_b200")], check=True)
    return capi.load()


def test_header_matches_binding():
    assert header_functions() == capi.exported_symbols()


def test_library_exports_every_declared_symbol(lib):
    for name in header_functions():
        assert hasattr(lib, name), name
    out = subprocess.run(["nm", "-D", "--defined-only", str(capi.LIB_PATH)],
                         capture_output=True, text=True, check=True).stdout
    exported = set(re.findall(r"\bT (pspml_\w+)", out))
    assert set(header_functions()) <= exported


def test_abi_version_and_no_device_paths(lib):
    assert lib.pspml_abi_version() == 2
    n = ctypes.c_int(-1)
    assert lib.pspml_device_count(ctypes.byref(n)) == capi.OK
    assert n.value >= 0


def test_errors_are_status_codes(lib):
    # null arguments come back as INVALID_ARG with a message, never a crash
    assert lib.pspml_ctx_create(0, 0, None) == capi.ERR_INVALID_ARG
    assert b"null" in lib.pspml_last_error()
    d = capi.OpDesc()
    d.kind = capi.OP_CONV2D
    assert lib.pspml_conv2d_s8(None, ctypes.byref(d), 1, None, None, None, None, None, None,
                               None) == capi.ERR_INVALID_ARG
    assert lib.pspml_model_create(None, None, 0, None, 0, 1, None) == capi.ERR_INVALID_ARG
    assert lib.pspml_forward(None, None, None, 1, None) == capi.ERR_INVALID_ARG
    assert lib.pspml_ctx_wait_selftest(None, 1000, 0) == capi.ERR_INVALID_ARG
    assert lib.pspml_model_fail_next(None, 1, capi.ERR_CUDA) == capi.ERR_INVALID_ARG


def test_timing_struct_layout():
    # double x3, int32 x3 (padded to 8): must match struct pspml_timing
    assert ctypes.sizeof(capi.Timing) == 40
    assert capi.Timing.rerun_shards.offset == 32


def test_pool_window_in_padding_rejected(lib):
    # A pooling window that lies entirely in the padding would average over
    # no input at all: rejected before any device work.
    d = capi.OpDesc()
    d.kind = capi.OP_AVERAGE_POOL2D
    d.in_h = d.in_w = 4
    d.in_c = d.out_c = 4
    d.kernel_h = d.kernel_w = 2
    d.stride_h = d.stride_w = 2
    d.pad_top = 2
    d.out_h = (4 + 2 - 2) // 2 + 1
    d.out_w = 2
    d.act_min, d.act_max = -128, 127
    st = lib.pspml_average_pool2d_s8(ctypes.c_void_p(1), ctypes.byref(d), 1,
                                     ctypes.c_void_p(16), ctypes.c_void_p(16), None)
    assert st == capi.ERR_INVALID_ARG
    assert b"padding" in lib.pspml_last_error()


def test_bad_descriptor_rejected_before_device_work(lib):
    d = capi.OpDesc()
    d.kind = capi.OP_CONV2D
    d.in_h = d.in_w = 8
    d.in_c = 4
    d.out_h = d.out_w = 7          # wrong for 3x3 / stride 1 / pad 1
    d.out_c = 4
    d.kernel_h = d.kernel_w = 3
    d.stride_h = d.stride_w = 1
    d.pad_top = d.pad_left = d.pad_bottom = d.pad_right = 1
    d.act_min, d.act_max = -128, 127
    st = lib.pspml_conv2d_s8(ctypes.c_void_p(1), ctypes.byref(d), 1, ctypes.c_void_p(16),
                             ctypes.c_void_p(16), None, ctypes.c_void_p(16),
                             ctypes.c_void_p(16), ctypes.c_void_p(16), None)
    assert st == capi.ERR_INVALID_ARG
    assert b"output size" in lib.pspml_last_error()
