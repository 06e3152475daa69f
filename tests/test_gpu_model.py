"""Whole-network parity on the B200: the compiled model (arena planner,
micro-batching, host-buffer pipeline, sharded and timed forwards) against
the oracle's network forward, bit-exact int8 logits."""
import ctypes

import numpy as np
import pytest

from pspml import capi, netspec

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def nets():
    return {c: netspec.BUILDERS[c]() for c in (0, 2, 3)}


def _device_forward(model, x, batch):
    import torch
    xi = torch.from_numpy(x.reshape(-1)).cuda()
    out = torch.full((batch * model.out_bytes,), 77, dtype=torch.int8, device="cuda")
    model.forward_device(xi.data_ptr(), out.data_ptr(), batch,
                         torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    return out.cpu().numpy().reshape(batch, -1)


@pytest.mark.parametrize("cfg,batch,micro", [(0, 37, 16), (0, 5, 64), (2, 5, 2), (3, 3, 2),
                                             (3, 4, 8)])
def test_network_device_forward_bit_exact(ctx, oracle_mod, nets, cfg, batch, micro):
    net = nets[cfg]
    descs, blob = net.descs_and_blob()
    x = net.make_input(batch)
    want = oracle_mod.net_forward_s8(descs, blob, x)
    model = capi.Model(ctx, descs, blob, micro)
    got = _device_forward(model, x, batch)
    ctx.check_device()
    assert np.array_equal(got, want), f"{np.count_nonzero(got != want)} logits differ"
    model.close()


def test_network_host_forward_and_sharded(ctx, oracle_mod, nets):
    import torch
    net = nets[3]
    descs, blob = net.descs_and_blob()
    batch = 6
    x = net.make_input(batch)
    want = oracle_mod.net_forward_s8(descs, blob, x)
    model = capi.Model(ctx, descs, blob, 2)
    hin = torch.from_numpy(x.reshape(-1).copy()).pin_memory()
    hout = torch.zeros(batch * net.out_elems, dtype=torch.int8).pin_memory()
    t = model.forward(hin.data_ptr(), hout.data_ptr(), batch)
    assert t.micro_batches == 3 and t.h2d_bytes == batch * net.in_elems
    assert np.array_equal(hout.numpy().reshape(batch, -1), want)
    hout.zero_()
    capi.forward_sharded([model], hin.data_ptr(), hout.data_ptr(), batch)
    assert np.array_equal(hout.numpy().reshape(batch, -1), want)
    model.close()


def test_forward_timed_reports_every_op(ctx, nets):
    import torch
    net = nets[0]
    descs, blob = net.descs_and_blob()
    model = capi.Model(ctx, descs, blob, 64)
    x = torch.from_numpy(net.make_input(64).reshape(-1)).cuda()
    out = torch.empty(64 * net.out_elems, dtype=torch.int8, device="cuda")
    ms = model.forward_timed(x.data_ptr(), out.data_ptr(), 64,
                             torch.cuda.current_stream().cuda_stream)
    assert len(ms) == len(net.layers) and all(v >= 0 for v in ms)
    model.close()


def test_arena_is_smaller_than_static_buffers(ctx, nets):
    net = nets[3]
    descs, blob = net.descs_and_blob()
    model = capi.Model(ctx, descs, blob, 4)
    static = 4 * sum(int(np.prod(l.out_shape)) for l in net.layers[:-1])
    assert model.arena_bytes < static
    model.close()


@pytest.mark.parametrize("B,K", [(1, 512), (1, 8192), (256, 2048), (256, 512)])
def test_fc_sweep_points(ctx, oracle_mod, B, K):
    net = netspec.build_fc_sweep(B, K)
    descs, blob = net.descs_and_blob()
    x = net.make_input(B)
    want = oracle_mod.net_forward_s8(descs, blob, x)
    model = capi.Model(ctx, descs, blob, B)
    got = _device_forward(model, x, B)
    assert np.array_equal(got, want)
    model.close()


def test_fc_sweep_largest_point_sampled_rows(ctx, oracle_mod):
    """B=16384, K=N=8192 on the GPU; the oracle checks 48 sampled rows."""
    B, K = 16384, 8192
    net = netspec.build_fc_sweep(B, K)
    descs, blob = net.descs_and_blob()
    x = net.make_input(B)
    model = capi.Model(ctx, descs, blob, B)
    got = _device_forward(model, x, B)
    rows = np.random.default_rng(0).choice(B, 48, replace=False)
    rows = np.concatenate([rows, [0, 127, 128, B - 1]])
    want = oracle_mod.net_forward_s8(descs, blob, x[rows])
    assert np.array_equal(got[rows], want)
    model.close()


def test_bad_model_rejected(ctx, nets):
    descs, blob = nets[0].descs_and_blob()
    bad = descs.copy()
    bad[1]["in_c"] = 9  # breaks the chain
    with pytest.raises(capi.PspmlError) as e:
        capi.Model(ctx, bad, blob, 4)
    assert e.value.status == capi.ERR_INVALID_ARG
    bad = descs.copy()
    bad[0]["filter_off"] = blob.nbytes  # outside the blob
    with pytest.raises(capi.PspmlError):
        capi.Model(ctx, bad, blob, 4)
