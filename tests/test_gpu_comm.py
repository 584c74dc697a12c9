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
            rt.comm_wait(device, 10000)
            assert torch.equal(out, t)
    finally:
        rt.comm_destroy(device)
    rt.comm_destroy(device)  # no communicator left: a no-op


_NEVER_JOINED = r"""
import sys, time
sys.path[:0] = [ROOT, ROOT + "/ml-reentry-mlir_b200"]
import torch
from gnnc.b200 import runtime as rt
from gnnc.b200._lib import ERR_TIMEOUT, GnncError

dev = torch.device("cuda", 0)
uid = rt.comm_unique_id(dev)
t0 = time.monotonic()
try:
    rt.comm_init(dev, uid, 0, 2, timeout_ms=3000)  # rank 1 never joins
    print("JOINED")
    sys.exit(1)
except GnncError as exc:
    waited = time.monotonic() - t0
    assert exc.status == ERR_TIMEOUT, exc
    print(f"TIMEOUT after {waited:.2f}s: {exc}")
# the context stays usable: a new one-rank communicator and a collective
rt.comm_init(dev, rt.comm_unique_id(dev), 0, 1, timeout_ms=30000)
x = torch.randn(256, 64, device=dev)
y = rt.allgather(x, torch.empty_like(x))
rt.comm_wait(dev, 10000)
assert torch.equal(x, y)
rt.comm_destroy(dev)
print(f"WAITED {waited:.3f}")
"""


@pytest.mark.timeout(240)
def test_comm_init_gives_up_when_a_rank_never_joins(device):
    """gnnc_comm_init_timeout: rank 0 of a two-rank communicator whose rank 1
    never joins returns GNNC_ERR_TIMEOUT shortly after its 3 s deadline (the
    non-blocking communicator is aborted), and the same context then joins a
    one-rank communicator and runs a collective. A fresh process with NVLS off:
    nothing runs on the GPU while the join is pending."""
    import subprocess

    env = dict(os.environ, NCCL_NVLS_ENABLE="0", CUDA_VISIBLE_DEVICES=str(device.index or 0))
    code = f"ROOT = {ROOT!r}\n" + _NEVER_JOINED
    t0 = time.monotonic()
    res = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True,
                         timeout=200)
    assert res.returncode == 0, res.stdout[-2000:] + res.stderr[-3000:]
    assert "TIMEOUT after" in res.stdout, res.stdout
    waited = float(res.stdout.split("WAITED")[1].split()[0])
    assert 3.0 <= waited < 15.0, waited
    assert time.monotonic() - t0 < 200


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
