"""The no-allocation fully-connected entry point against the regular one.

pspml_fully_connected_s8_noalloc serves callers that cannot allocate device
memory (CUDA graph capture, fixed memory budgets, caller-owned buffers): it
takes no context and keeps its scratch in a fixed array inside the library.
Its output must equal pspml_fully_connected_s8's, bit for bit (integer
arithmetic), on consecutive calls that reuse that shared scratch.  This file
is collected last so that a run stopping at the first failure has already
run every other test; it also passes when run alone in a fresh process.
"""
import ctypes

import numpy as np
import pytest

from gpu_helpers import make_desc, random_quant
from pspml import capi

pytestmark = pytest.mark.gpu


def _fc_desc(K, N, zp_in=-3, zp_out=5, act=(5, 127)):
    return make_desc(kind=capi.OP_FULLY_CONNECTED, in_h=1, in_w=1, in_c=K, out_h=1, out_w=1,
                     out_c=N, zp_in=zp_in, zp_out=zp_out, act_min=act[0], act_max=act[1])


def _run_both(ctx, d, B, seed, mode="calibrated"):
    import torch
    r = np.random.default_rng(seed)
    K, N = int(d["in_c"]), int(d["out_c"])
    x = torch.from_numpy(r.integers(-128, 128, (B, K)).astype(np.int8).reshape(-1)).cuda()
    w = torch.from_numpy(r.integers(-127, 128, (N, K)).astype(np.int8).reshape(-1)).cuda()
    b, m, s = (torch.from_numpy(a).cuda() for a in random_quant(r, N, mode))
    stream = torch.cuda.current_stream().cuda_stream
    ds = capi.desc_struct(d)
    ref = torch.empty(B * N, dtype=torch.int8, device="cuda")
    capi.call("pspml_fully_connected_s8", ctx.handle, ctypes.byref(ds), B, x.data_ptr(),
              w.data_ptr(), b.data_ptr(), m.data_ptr(), s.data_ptr(), ref.data_ptr(), stream)
    got = torch.full((B * N,), 99, dtype=torch.int8, device="cuda")
    capi.call("pspml_fully_connected_s8_noalloc", ctypes.byref(ds), B, x.data_ptr(),
              w.data_ptr(), b.data_ptr(), m.data_ptr(), s.data_ptr(), got.data_ptr(), stream)
    torch.cuda.synchronize()
    return ref.cpu().numpy(), got.cpu().numpy()


@pytest.fixture(scope="module")
def fc_ctx():
    import torch
    torch.cuda.init()
    c = capi.Context(0)
    yield c
    c.close()


def test_noalloc_matches_regular_entry_point_on_consecutive_calls(fc_ctx):
    # Two calls in a row with different shapes and quantisation: the second
    # reuses the scratch the first one filled.
    cases = [(_fc_desc(512, 3337), 257, 1, "calibrated"),
             (_fc_desc(784, 10, zp_in=-128, zp_out=0, act=(-128, 127)), 33, 2, "extreme")]
    for d, B, seed, mode in cases:
        ref, got = _run_both(fc_ctx, d, B, seed, mode)
        assert np.array_equal(ref, got), f"{np.count_nonzero(ref != got)} outputs differ"


def test_noalloc_cuda_core_path_twice(fc_ctx):
    # K % 16 != 0 takes the CUDA-core FC kernel; run it twice in a row.
    d = _fc_desc(100, 7)
    for seed in (3, 4):
        ref, got = _run_both(fc_ctx, d, 5, seed)
        assert np.array_equal(ref, got)


def test_noalloc_rejects_ops_beyond_its_scratch():
    d = _fc_desc(64, 20000)
    ds = capi.desc_struct(d)
    lib = capi.load()
    st = lib.pspml_fully_connected_s8_noalloc(ctypes.byref(ds), 1, ctypes.c_void_p(256),
                                              ctypes.c_void_p(256), None, ctypes.c_void_p(256),
                                              ctypes.c_void_p(256), ctypes.c_void_p(256), None)
    assert st == capi.ERR_INVALID_ARG
    assert b"no-allocation" in lib.pspml_last_error()
