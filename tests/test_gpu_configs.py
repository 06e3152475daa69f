"""Parity of the benchmark configurations on the B200, bit-exact int8 against
the oracle:

* config 1: every point of the FullyConnected sweep, B in {1, 256, 16384}
  and K = N in {512, 2048, 8192}.  The B = 16384 points check all rows at
  K = 512 and at least 512 sampled rows otherwise, always including the
  edges of the 128- and 256-row tiles and the last row.
* config 2: the whole network over a batch that spans several
  micro-batches (a ragged last one included), and its stage-2/3 conv layers
  at their real shapes with their real weights.
"""
import numpy as np
import pytest

from pspml import capi, netspec

pytestmark = pytest.mark.gpu


def _device_forward(model, x, batch):
    import torch
    xi = torch.from_numpy(np.ascontiguousarray(x).reshape(-1)).cuda()
    out = torch.full((batch * model.out_bytes,), 77, dtype=torch.int8, device="cuda")
    model.forward_device(xi.data_ptr(), out.data_ptr(), batch,
                         torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    return out.cpu().numpy().reshape(batch, -1)


def _tile_edge_rows(B):
    edges = set()
    for t in (128, 256):
        for k in range(t, B, t * 7):
            edges.update((k - 1, k))
    edges.update((0, 1, B - 2, B - 1))
    return sorted(r for r in edges if 0 <= r < B)


@pytest.mark.parametrize("B,K", [(b, k) for b in (1, 256) for k in (512, 2048, 8192)])
def test_fc_sweep_point_all_rows(ctx, oracle_mod, B, K):
    net = netspec.build_fc_sweep(B, K)
    descs, blob = net.descs_and_blob()
    x = net.make_input(B)
    model = capi.Model(ctx, descs, blob, B)
    got = _device_forward(model, x, B)
    ctx.check_device()
    model.close()
    want = oracle_mod.net_forward_s8(descs, blob, x)
    assert np.array_equal(got, want), f"{np.count_nonzero(got != want)} outputs differ"


@pytest.mark.parametrize("K,rows", [(512, None), (2048, 1024), (8192, 512)])
def test_fc_sweep_b16384(ctx, oracle_mod, K, rows):
    B = 16384
    net = netspec.build_fc_sweep(B, K)
    descs, blob = net.descs_and_blob()
    x = net.make_input(B)
    model = capi.Model(ctx, descs, blob, B)
    got = _device_forward(model, x, B)
    ctx.check_device()
    model.close()
    if rows is None:
        sel = np.arange(B)
    else:
        edges = _tile_edge_rows(B)
        rng = np.random.default_rng(K)
        rest = rng.choice(np.setdiff1d(np.arange(B), edges), rows - len(edges), replace=False)
        sel = np.sort(np.concatenate([edges, rest]))
        assert len(sel) >= rows
    want = oracle_mod.net_forward_s8(descs, blob, x[sel])
    assert np.array_equal(got[sel], want), f"{np.count_nonzero(got[sel] != want)} outputs differ"


def test_config2_network_over_several_micro_batches(ctx, oracle_mod):
    net = netspec.build_config2()
    descs, blob = net.descs_and_blob()
    batch = 11  # micro-batches of 4, 4 and 3
    x = net.make_input(batch, tag="multi-micro")
    model = capi.Model(ctx, descs, blob, 4)
    got = _device_forward(model, x, batch)
    ctx.check_device()
    model.close()
    want = oracle_mod.net_forward_s8(descs, blob, x)
    assert np.array_equal(got, want), f"{np.count_nonzero(got != want)} logits differ"


def _single_layer_net(net, name):
    layer = next(l for l in net.layers if l.name == name)
    return netspec.Network(f"{net.name}/{name}", [layer], layer.in_shape, layer.s_in,
                           layer.zp_in, input_kind="uniform_int8")


@pytest.mark.parametrize("name,batch", [("s2a", 24), ("s2b", 24), ("s3a", 48), ("s3b", 48),
                                        ("s1b", 6)])
def test_config2_conv_layer_at_real_shape(ctx, oracle_mod, name, batch):
    one = _single_layer_net(netspec.build_config2(), name)
    descs, blob = one.descs_and_blob()
    x = one.make_input(batch, tag="layer")
    model = capi.Model(ctx, descs, blob, batch)
    got = _device_forward(model, x, batch)
    ctx.check_device()
    model.close()
    want = oracle_mod.net_forward_s8(descs, blob, x)
    assert np.array_equal(got, want), f"{np.count_nonzero(got != want)} outputs differ"
