"""Failure detection on the B200, without faulting or hanging the GPU.

* A kernel's bounded wait that runs out: pspml_ctx_wait_selftest waits, with
  the tensor-core kernels' own bounded-wait primitive, on an mbarrier that
  nothing arrives on; after a short limit it records a code in the context's
  device error word and returns.  pspml_ctx_check_device then reports
  PSPML_ERR_DEVICE_WAIT and the context stays usable.
* The host watchdog: a forward whose deadline passes returns
  PSPML_ERR_TIMEOUT while its device work runs to completion on its own.
* A failed device in a sharded forward (injected on the host with
  pspml_model_fail_next): its slice is re-run on the devices that succeeded.
"""
import ctypes
import time

import numpy as np
import pytest

from pspml import capi, netspec

pytestmark = pytest.mark.gpu


def test_bounded_wait_expiry_reports_device_wait(ctx, oracle_mod):
    ctx.check_device()  # starts clear
    t0 = time.perf_counter()
    ctx.wait_selftest(50_000, signal=False)  # nothing arrives: gives up after ~50 ms
    waited = time.perf_counter() - t0
    assert 0.04 < waited < 5.0
    with pytest.raises(capi.PspmlError) as e:
        ctx.check_device()
    assert e.value.status == capi.ERR_DEVICE_WAIT
    ctx.check_device()  # reading it cleared the word
    ctx.wait_selftest(50_000, signal=True)  # a signalled wait completes
    ctx.check_device()
    # The context still runs work, bit-exact.
    net = netspec.build_config0()
    descs, blob = net.descs_and_blob()
    x = net.make_input(4)
    model = capi.Model(ctx, descs, blob, 4)
    import torch
    xi = torch.from_numpy(x.reshape(-1)).cuda()
    out = torch.empty(4 * net.out_elems, dtype=torch.int8, device="cuda")
    model.forward_device(xi.data_ptr(), out.data_ptr(), 4, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    ctx.check_device()
    assert np.array_equal(out.cpu().numpy().reshape(4, -1), oracle_mod.net_forward_s8(descs, blob, x))
    model.close()


def test_wait_selftest_rejects_bad_limits(ctx):
    for bad in (0, -5, 10_000_001):
        with pytest.raises(capi.PspmlError) as e:
            ctx.wait_selftest(bad, signal=True)
        assert e.value.status == capi.ERR_INVALID_ARG


def test_host_watchdog_times_out_then_recovers(oracle_mod):
    import torch
    net = netspec.build_config3()
    descs, blob = net.descs_and_blob()
    batch = 2048
    x = net.make_input(batch)
    with capi.Context(0) as c:
        model = capi.Model(c, descs, blob, 512)
        hin = torch.from_numpy(x.reshape(-1).copy()).pin_memory()
        hout = torch.zeros(batch * net.out_elems, dtype=torch.int8).pin_memory()
        c.set_timeout_ms(1)  # far shorter than copying and running 2048 samples
        with pytest.raises(capi.PspmlError) as e:
            model.forward(hin.data_ptr(), hout.data_ptr(), batch)
        assert e.value.status == capi.ERR_TIMEOUT
        # The device work ran on; wait for it before reusing the buffers.
        torch.cuda.synchronize()
        c.set_timeout_ms(60_000)
        hout.zero_()
        model.forward(hin.data_ptr(), hout.data_ptr(), batch)
        c.check_device()
        got = hout.numpy().reshape(batch, -1)
        rows = [0, 1, 511, 512, 1500, batch - 1]
        assert np.array_equal(got[rows], oracle_mod.net_forward_s8(descs, blob, x[rows]))
        model.close()


def test_sharded_forward_reruns_a_failed_shard(ctx, oracle_mod):
    import torch
    net = netspec.build_config0()
    descs, blob = net.descs_and_blob()
    batch = 50
    x = net.make_input(batch)
    want = oracle_mod.net_forward_s8(descs, blob, x)
    models = [capi.Model(ctx, descs, blob, 8) for _ in range(3)]
    hin = torch.from_numpy(x.reshape(-1).copy()).pin_memory()
    hout = torch.zeros(batch * net.out_elems, dtype=torch.int8).pin_memory()
    models[1].fail_next(1, capi.ERR_CUDA)
    t = capi.forward_sharded(models, hin.data_ptr(), hout.data_ptr(), batch)
    assert t.rerun_shards == 1 and t.devices == 3
    assert np.array_equal(hout.numpy().reshape(batch, -1), want)
    # Nothing left to inject: a plain run re-runs nothing.
    hout.zero_()
    t = capi.forward_sharded(models, hin.data_ptr(), hout.data_ptr(), batch)
    assert t.rerun_shards == 0
    assert np.array_equal(hout.numpy().reshape(batch, -1), want)
    # Every device failing is an error, carrying the failure's status.
    for m in models:
        m.fail_next(1, capi.ERR_OOM)
    with pytest.raises(capi.PspmlError) as e:
        capi.forward_sharded(models, hin.data_ptr(), hout.data_ptr(), batch)
    assert e.value.status == capi.ERR_OOM
    # A timed-out shard is not re-run (its device may still write its slice).
    models[2].fail_next(1, capi.ERR_TIMEOUT)
    with pytest.raises(capi.PspmlError) as e:
        capi.forward_sharded(models, hin.data_ptr(), hout.data_ptr(), batch)
    assert e.value.status == capi.ERR_TIMEOUT
    torch.cuda.synchronize()
    for m in models:
        m.close()
