"""Collectives through the C ABI: gnnc_comm_unique_id / gnnc_comm_init /
gnnc_allgather / gnnc_comm_destroy.

On one GPU a one-rank communicator checks the whole call sequence (the
all-gather of one rank is a copy) and the argument errors; with two GPUs two
processes gather each other's rows, rank order kept, bit for bit."""

from __future__ import annotations

import os
import sys
import time

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_one_rank_communicator(device):
    from gnnc.b200 import runtime as rt
    from gnnc.b200._lib import GnncInvalidArgument

    x = torch.randn(1000, 104, device=device).to(torch.bfloat16)
    with pytest.raises(GnncInvalidArgument, match="no communicator"):
        rt.allgather(x, torch.empty_like(x))
    uid = rt.comm_unique_id(device)
    assert len(uid) == rt.COMM_ID_BYTES
    rt.comm_init(device, uid, 0, 1)
    try:
        with pytest.raises(GnncInvalidArgument, match="already has a communicator"):
            rt.comm_init(device, uid, 0, 1)
        for t in (x, torch.randn(333, 4, device=device)):
            out = rt.allgather(t, torch.empty_like(t))
            rt.Context.get(device).synchronize()
            assert torch.equal(out, t)
    finally:
        rt.comm_destroy(device)
    rt.comm_destroy(device)  # no communicator left: a no-op


def _rank(rank, world, path, out_dir):
    sys.path[:0] = [ROOT, os.path.join(ROOT, "ml-reentry-mlir_b200")]
    from gnnc.b200 import runtime as rt

    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    if rank == 0:
        uid = rt.comm_unique_id(dev)
        with open(path + ".tmp", "wb") as f:
            f.write(uid)
        os.replace(path + ".tmp", path)
    else:
        for _ in range(600):  # at most a minute
            if os.path.exists(path):
                break
            time.sleep(0.1)
        with open(path, "rb") as f:
            uid = f.read()
    rt.comm_init(dev, uid, rank, world)
    g = torch.Generator().manual_seed(rank)
    mine = torch.randn(500, 104, generator=g).to(torch.bfloat16)
    recv = torch.empty((world * 500, 104), dtype=torch.bfloat16, device=dev)
    rt.allgather(mine.to(dev), recv)
    rt.Context.get(dev).synchronize()
    torch.save(recv.cpu(), os.path.join(out_dir, f"r{rank}.pt"))
    rt.comm_destroy(dev)


@pytest.mark.timeout(300)
def test_two_gpu_allgather(device, tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    world = 2
    mp.spawn(_rank, args=(world, str(tmp_path / "uid"), str(tmp_path)), nprocs=world, join=True)
    want = torch.cat([torch.randn(500, 104, generator=torch.Generator().manual_seed(r)).to(torch.bfloat16)
                      for r in range(world)])
    for r in range(world):
        assert torch.equal(torch.load(tmp_path / f"r{r}.pt"), want)
