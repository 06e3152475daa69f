"""Batch sharding across ranks, exercised with world-size-2 gloo processes on
the CPU: every rank runs its contiguous slice (here through the oracle, the
CPU stand-in for a device), and the slices concatenated in rank order equal
the single-process result.  The product path has no collective; the gather
below only checks the result."""
import os
import socket

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from pspml import shard


def test_slices_cover_batch_exactly():
    for batch in (0, 1, 7, 262144, 262143):
        for world in (1, 2, 3, 4, 8):
            sl = shard.all_slices(batch, world)
            assert sl[0][0] == 0 and sl[-1][1] == batch
            for (a, b), (c, d) in zip(sl, sl[1:]):
                assert b == c and a <= b and c <= d
            assert max(b - a for a, b in sl) == -(-batch // world) if batch else True


def test_bad_shard_arguments():
    with pytest.raises(ValueError):
        shard.slice_for(10, 0, 0)
    with pytest.raises(ValueError):
        shard.slice_for(10, 2, 2)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, batch, q):
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parents[1]
    sys.path.insert(0, str(root / "psp-ml_b200"))
    sys.path.insert(0, str(root))
    import torch
    from oracle import oracle as orc
    from pspml import netspec, shard as sh
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        net = netspec.build_config0()
        descs, blob = net.descs_and_blob()
        x = net.make_input(batch)
        a, b = sh.slice_for(batch, world, rank)
        mine = orc.net_forward_s8(descs, blob, x[a:b], threads=1) if b > a else \
            np.zeros((0, net.out_elems), np.int8)
        per = -(-batch // world)
        padded = np.zeros((per, net.out_elems), np.int8)
        padded[: b - a] = mine
        gathered = [torch.zeros(per, net.out_elems, dtype=torch.int8) for _ in range(world)]
        dist.all_gather(gathered, torch.from_numpy(padded))
        if rank == 0:
            parts = [g.numpy()[: e - s] for g, (s, e) in zip(gathered, sh.all_slices(batch, world))]
            full = orc.net_forward_s8(descs, blob, x, threads=1)
            q.put(bool(np.array_equal(np.concatenate(parts), full)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("batch", [9, 16])
def test_two_rank_sharded_forward_matches_single(batch):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, batch, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert q.get(timeout=5) is True
