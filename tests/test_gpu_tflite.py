"""A .tflite int8 model imported through pspml.tflite runs on the B200
bit-exact against the oracle: the config networks are written as TFLite
files, read back, lowered to op descriptors and run through the C-ABI
model."""
import numpy as np
import pytest

from pspml import capi, netspec, tflite

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("cfg,batch", [(0, 33), (3, 3)])
def test_imported_tflite_model_bit_exact(ctx, oracle_mod, cfg, batch):
    import torch
    data = tflite.write_network(netspec.BUILDERS[cfg]())
    net = tflite.to_network(tflite.load(data), name=f"imported_cfg{cfg}")
    descs, blob = net.descs_and_blob()
    x = netspec.BUILDERS[cfg]().make_input(batch)
    want = oracle_mod.net_forward_s8(descs, blob, x)
    model = capi.Model(ctx, descs, blob, batch)
    xi = torch.from_numpy(x.reshape(-1)).cuda()
    out = torch.empty(batch * net.out_elems, dtype=torch.int8, device="cuda")
    model.forward_device(xi.data_ptr(), out.data_ptr(), batch,
                         torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    ctx.check_device()
    got = out.cpu().numpy().reshape(batch, -1)
    model.close()
    assert np.array_equal(got, want), f"{np.count_nonzero(got != want)} logits differ"
