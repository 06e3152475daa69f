"""Model creation on a busy GPU, bit-exact against the oracle.

A model uploads its weight blob and then builds its requantisation and
folded-bias tables with kernels on the context's stream.  Both steps must
be ordered on that stream: an upload issued on another stream may still be
in flight when the table kernels read the multipliers, and the model then
computes with zero tables (every output at the output zero point).  The
copy engine is kept busy here with a large pinned host-to-device copy on a
side stream while each model is created, which delays any upload that is
not ordered before the table kernels.
"""
import numpy as np
import pytest

from pspml import capi, netspec

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("B,K", [(4, 2048), (256, 2048)])
def test_model_tables_follow_the_weight_upload(ctx, oracle_mod, B, K):
    import torch
    net = netspec.build_fc_sweep(B, K)
    descs, blob = net.descs_and_blob()
    x = net.make_input(B)
    want = oracle_mod.net_forward_s8(descs, blob, x)
    host = torch.empty(256 << 20, dtype=torch.int8).pin_memory()
    dev = torch.empty_like(host, device="cuda")
    side = torch.cuda.Stream()
    xi = torch.from_numpy(np.ascontiguousarray(x).reshape(-1)).cuda()
    torch.cuda.synchronize()
    for _ in range(3):
        with torch.cuda.stream(side):
            dev.copy_(host, non_blocking=True)
        model = capi.Model(ctx, descs, blob, B)
        out = torch.full((B * model.out_bytes,), 77, dtype=torch.int8, device="cuda")
        model.forward_device(xi.data_ptr(), out.data_ptr(), B,
                             torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        ctx.check_device()
        model.close()
        got = out.cpu().numpy().reshape(B, -1)
        assert np.array_equal(got, want), f"{np.count_nonzero(got != want)} outputs differ"
