"""The no-allocation fully-connected entry point against the regular one and
the oracle.

pspml_fully_connected_s8_noalloc serves callers that cannot allocate device
memory (code running under CUDA graph capture, hosts whose device memory
budget is fixed at start-up, callers that pass only buffers they already
own): it takes no context and keeps its scratch in a fixed array inside the
library.  Its output must equal pspml_fully_connected_s8's and the oracle's,
bit for bit (integer arithmetic), on consecutive calls that reuse that
shared scratch, and a call after the first must leave the device's free
memory unchanged.  This file is collected last so that a run stopping at the
first failure has already run every other test; it also passes when run
alone in a fresh process.
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


class _Case:
    """One FC op's tensors on the device, allocated before any measured call."""

    def __init__(self, d, B, seed, mode="calibrated"):
        import torch
        r = np.random.default_rng(seed)
        K, N = int(d["in_c"]), int(d["out_c"])
        self.d, self.B, self.N = d, B, N
        self.x_h = r.integers(-128, 128, (B, K)).astype(np.int8)
        self.w_h = r.integers(-127, 128, (N, K)).astype(np.int8)
        self.q_h = random_quant(r, N, mode)
        self.x = torch.from_numpy(self.x_h.reshape(-1)).cuda()
        self.w = torch.from_numpy(self.w_h.reshape(-1)).cuda()
        self.b, self.m, self.s = (torch.from_numpy(a).cuda() for a in self.q_h)
        self.ref = torch.empty(B * N, dtype=torch.int8, device="cuda")
        self.got = torch.full((B * N,), 99, dtype=torch.int8, device="cuda")
        self.ds = capi.desc_struct(d)

    def args(self, out):
        return (ctypes.byref(self.ds), self.B, self.x.data_ptr(), self.w.data_ptr(),
                self.b.data_ptr(), self.m.data_ptr(), self.s.data_ptr(), out.data_ptr())

    def run_noalloc(self, stream):
        capi.call("pspml_fully_connected_s8_noalloc", *self.args(self.got), stream)

    def run_regular(self, ctx, stream):
        capi.call("pspml_fully_connected_s8", ctx.handle, *self.args(self.ref), stream)

    def oracle(self, orc):
        b, m, s = self.q_h
        return orc.op_s8(self.d, self.B, self.x_h, self.w_h, b, m, s)


@pytest.fixture(scope="module")
def fc_ctx():
    import torch
    torch.cuda.init()
    c = capi.Context(0)
    yield c
    c.close()


def _check(case, orc):
    import torch
    torch.cuda.synchronize()
    capi.call("pspml_noalloc_check_device")
    got = case.got.cpu().numpy()
    assert np.array_equal(got, case.ref.cpu().numpy()), \
        f"{np.count_nonzero(got != case.ref.cpu().numpy())} outputs differ from the regular call"
    assert np.array_equal(got, case.oracle(orc)), "outputs differ from the oracle"


def test_noalloc_matches_regular_entry_point_and_oracle_on_consecutive_calls(fc_ctx, oracle_mod):
    import torch
    stream = torch.cuda.current_stream().cuda_stream
    # Two calls in a row with different shapes and quantisation: the second
    # reuses the scratch the first one filled.
    cases = [_Case(_fc_desc(512, 3337), 257, 1, "calibrated"),
             _Case(_fc_desc(784, 10, zp_in=-128, zp_out=0, act=(-128, 127)), 33, 2, "extreme")]
    for c in cases:
        c.run_regular(fc_ctx, stream)
        c.run_noalloc(stream)
        _check(c, oracle_mod)


def test_noalloc_cuda_core_path_twice(fc_ctx, oracle_mod):
    import torch
    stream = torch.cuda.current_stream().cuda_stream
    # K % 16 != 0 takes the CUDA-core FC kernel; run it twice in a row.
    for seed in (3, 4):
        c = _Case(_fc_desc(100, 7), 5, seed)
        c.run_regular(fc_ctx, stream)
        c.run_noalloc(stream)
        _check(c, oracle_mod)


def test_noalloc_calls_leave_device_free_memory_unchanged(oracle_mod):
    import torch
    stream = torch.cuda.current_stream().cuda_stream
    cases = [_Case(_fc_desc(512, 1024), 300, 5), _Case(_fc_desc(256, 64), 17, 6)]
    cases[0].run_noalloc(stream)  # the first call on the device does its set-up
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    for _ in range(3):
        for c in cases:
            c.run_noalloc(stream)
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0, f"device free memory moved by {free0 - free1} bytes"
    capi.call("pspml_noalloc_check_device")
    for c in cases:
        b, m, s = c.q_h
        want = oracle_mod.op_s8(c.d, c.B, c.x_h, c.w_h, b, m, s)
        assert np.array_equal(c.got.cpu().numpy(), want)


def test_noalloc_rejects_ops_beyond_its_scratch():
    d = _fc_desc(64, 20000)
    ds = capi.desc_struct(d)
    lib = capi.load()
    st = lib.pspml_fully_connected_s8_noalloc(ctypes.byref(ds), 1, ctypes.c_void_p(256),
                                              ctypes.c_void_p(256), None, ctypes.c_void_p(256),
                                              ctypes.c_void_p(256), ctypes.c_void_p(256), None)
    assert st == capi.ERR_INVALID_ARG
    assert b"no-allocation" in lib.pspml_last_error()
