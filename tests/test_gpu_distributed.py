"""Row-partitioned whole-model forward (gnnc.b200.distributed) vs one process.

Two ranks run as two processes on cuda:0 (a gloo group with host fences; the
CUDA IPC mappings work between processes of one device), so the test needs one
GPU. Each rank's output rows must equal the same rows of the single-process
executable bit for bit: every row is projected and aggregated by the same
kernels on the same values; so must every batch of a pipelined stream
(run_stream). The models cover both exchange sides (input rows
for 100 -> 4x64 and 256 -> 256, projected rows for 256 -> 47), GCN, GAT and
SAGE, bf16 features, rows split across CTAs.
"""

from __future__ import annotations

import os
import socket
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs(model_name):
    from gnnc.examples.synthetic import config_model_edges
    from gnnc.examples.util import normalized_csr_adj

    n = 20_000
    ei = config_model_edges(n, 150_000, 2.1, seed=7)
    # a heavy destination (split across CTAs)
    hub = torch.stack([torch.randint(0, n, (9000,), generator=torch.Generator().manual_seed(1)),
                       torch.full((9000,), 11)])
    ei = torch.cat([ei, hub], 1)
    x = torch.randn(n, 100, generator=torch.Generator().manual_seed(2)).to(torch.bfloat16)
    graph = ei if model_name == "gat" else normalized_csr_adj(ei, n)
    return x, graph


def _model(model_name):
    from gnnc.examples.models import gat, gcn, sage

    if model_name == "gat":
        return gat.Model(100, 64, 47, heads=4, num_layers=3).eval()
    mod = gcn if model_name == "gcn" else sage
    return mod.Model(100, 256, 47, num_layers=3).eval()


def _rank(rank, world, port, out_dir, model_name):
    sys.path[:0] = [ROOT, os.path.join(ROOT, "ml-reentry-mlir_b200")]
    import torch.distributed as dist

    from gnnc.b200 import partition as P
    from gnnc.b200.distributed import distribute
    from gnnc.compile import compile_executable

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world)
    x, graph = _inputs(model_name)
    model = _model(model_name)
    exe, _ = compile_executable(model, (x, graph), target="b200")
    dexe = distribute(exe)
    modes = dexe.exchange_modes()
    rr = P.row_range(x.size(0), world, rank)
    outs = [dexe(x[rr.begin : rr.end], graph) for _ in range(2)]  # twice: buffers reused
    ref = exe(x, graph)[0][rr.begin : rr.end]
    # a stream of three different batches, the first layer's exchange pipelined
    xs = [x, (x.float() * 0.5).to(x.dtype), -x]
    stream = [o.cpu() for o in dexe.run_stream((xb[rr.begin : rr.end] for xb in xs), graph)]
    stream_ref = [exe(xb, graph)[0][rr.begin : rr.end] for xb in xs]
    torch.save({"outs": outs, "ref": ref, "modes": modes, "stream": stream,
                "stream_ref": stream_ref}, os.path.join(out_dir, f"r{rank}.pt"))
    dist.barrier()
    dexe.close()
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.timeout(600)
@pytest.mark.parametrize("model_name", ["gat", "gcn", "sage"])
def test_two_rank_forward_matches_single_process(device, tmp_path, model_name):
    import torch.multiprocessing as mp

    world = 2
    mp.spawn(_rank, args=(world, _free_port(), str(tmp_path), model_name), nprocs=world,
             join=True)
    for r in range(world):
        got = torch.load(tmp_path / f"r{r}.pt")
        assert got["modes"] == ["input", "input", "output"]
        for out in got["outs"]:
            assert out.shape == got["ref"].shape
            assert torch.equal(out, got["ref"]), f"rank {r}: max diff {(out - got['ref']).abs().max()}"
        assert len(got["stream"]) == 3
        for k, (out, ref) in enumerate(zip(got["stream"], got["stream_ref"], strict=True)):
            assert torch.equal(out, ref), f"rank {r}, batch {k}: max diff {(out - ref).abs().max()}"
        assert not torch.equal(got["stream"][0], got["stream"][2])
