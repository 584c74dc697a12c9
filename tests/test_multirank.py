"""Destination-row partitioning across ranks (world size 2, gloo, CPU).

Output exchange: each rank takes its row range and CSR slice
(gnnc.b200.partition), projects its own rows into its slot of the gathered
table, all-gathers h and a_src, and aggregates its rows. Input exchange: each
rank holds the input rows of its blocks, all-gathers X piece by piece,
projects every row and aggregates its own. Either way the stitched result must
equal the single-process layer. The aggregation arithmetic here is the CPU
oracle's; the logic under test is the partition / slot / all-gather
bookkeeping the GPU bench uses unchanged.
"""

from __future__ import annotations

import os
import socket
import sys

import numpy as np
import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _problem(n=301, H=2, C=3, K=5):
    from oracle import gnn_oracle as O

    g = torch.Generator().manual_seed(11)
    ei = torch.randint(0, n, (2, 2500), generator=g)
    hub = torch.stack([torch.randint(0, n, (400,), generator=g), torch.full((400,), 7)])
    ei = torch.cat([ei, hub], 1)
    rowptr, col, _ = O.csr_from_coo(ei.numpy(), n, self_loops=True, dedupe=False)
    x = torch.randn(n, K, generator=g, dtype=torch.float64)
    W = torch.randn(H * C, K, generator=g, dtype=torch.float64)
    a_s = torch.randn(H * C, generator=g, dtype=torch.float64)
    a_d = torch.randn(H * C, generator=g, dtype=torch.float64)
    return torch.from_numpy(rowptr), torch.from_numpy(col), x, W, a_s, a_d, H, C


def _rank_main(rank, world, port, out_dir):
    sys.path[:0] = [ROOT, os.path.join(ROOT, "ml-reentry-mlir_b200")]
    import torch.distributed as dist

    from gnnc.b200 import partition as P
    from oracle import gnn_oracle as O

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world)
    rowptr, col, x, W, a_s, a_d, H, C = _problem()
    n = x.size(0)
    rr = P.row_range(n, world, rank)
    rowptr_l, col_l = P.local_csr(rowptr, col, rr)
    table = P.gathered_table(rr, H * C, torch.float64, "cpu")
    a_tab = P.gathered_table(rr, H, torch.float64, "cpu")
    h = x[rr.begin : rr.end] @ W.t()
    P.my_rows(table, rr).copy_(h)
    P.my_rows(a_tab, rr).copy_((h.view(-1, H, C) * a_s.view(1, H, C)).sum(-1))
    adst_l = (h.view(-1, H, C) * a_d.view(1, H, C)).sum(-1)
    P.all_gather_rows(table, rr)
    P.all_gather_rows(a_tab, rr)
    out = O.gat_rows_fp64(rowptr_l, col_l, table[:n], a_tab[:n], adst_l, H)
    np.save(os.path.join(out_dir, f"rank{rank}.npy"), out.numpy())
    dist.barrier()
    dist.destroy_process_group()


def _rank_main_blocks(rank, world, port, out_dir, chunks):
    sys.path[:0] = [ROOT, os.path.join(ROOT, "ml-reentry-mlir_b200")]
    import torch.distributed as dist

    from gnnc.b200 import partition as P
    from oracle import gnn_oracle as O

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world)
    rowptr, col, x, W, a_s, a_d, H, C = _problem()
    n = x.size(0)
    rb = P.row_blocks(n, world, rank, chunks)
    rowptr_l, col_l = P.local_csr_blocks(rowptr, col, rb)
    ids = rb.node_ids()
    x_loc = P.local_blocks(rb, x.size(1), torch.float64, "cpu")
    x_loc[: rb.count] = x[ids]
    table = P.input_table(rb, x.size(1), torch.float64, "cpu")
    for c in range(rb.chunks):
        P.gather_piece(table, x_loc, rb, c)
    h = table @ W.t()
    asrc = (h.view(-1, H, C) * a_s.view(1, H, C)).sum(-1)
    adst = (h.view(-1, H, C) * a_d.view(1, H, C)).sum(-1)
    out = O.gat_rows_fp64(rowptr_l, col_l, h[:n], asrc[:n], P.owned_rows(adst, rb), H)
    np.save(os.path.join(out_dir, f"rank{rank}.npy"), out.numpy())
    np.save(os.path.join(out_dir, f"ids{rank}.npy"), ids.numpy())
    dist.barrier()
    dist.destroy_process_group()


def test_row_blocks_cover_every_row_once():
    from gnnc.b200 import partition as P

    for n in (1, 7, 8, 301, 1000):
        for world in (1, 2, 3, 8):
            for chunks in (1, 2, 4):
                blocks = [P.row_blocks(n, world, r, chunks) for r in range(world)]
                ids = torch.cat([b.node_ids() for b in blocks]).sort().values
                assert torch.equal(ids, torch.arange(n))
                for b in blocks:
                    # owned rows are the prefix of the local order
                    local = torch.arange(b.padded_rows).view(chunks, world, -1)[:, b.rank].reshape(-1)
                    assert torch.equal(local[: b.count], b.node_ids())
    # one chunk is the contiguous row range
    for r in range(3):
        b, rr = P.row_blocks(1000, 3, r), P.row_range(1000, 3, r)
        assert b.block(0) == (rr.begin, rr.end)


@pytest.mark.timeout(180)
def test_two_rank_gloo_input_exchange_matches_single_process(tmp_path):
    import torch.multiprocessing as mp

    from oracle import gnn_oracle as O

    world = 2
    mp.spawn(_rank_main_blocks, args=(world, _free_port(), str(tmp_path), 3), nprocs=world,
             join=True)
    got = np.concatenate([np.load(tmp_path / f"rank{r}.npy") for r in range(world)])
    ids = np.concatenate([np.load(tmp_path / f"ids{r}.npy") for r in range(world)])
    rowptr, col, x, W, a_s, a_d, H, C = _problem()
    h = x @ W.t()
    asrc = (h.view(-1, H, C) * a_s.view(1, H, C)).sum(-1)
    adst = (h.view(-1, H, C) * a_d.view(1, H, C)).sum(-1)
    ref = O.gat_rows_fp64(rowptr, col, h, asrc, adst, H).numpy()
    np.testing.assert_allclose(got, ref[ids], rtol=1e-12, atol=1e-12)


def test_row_range_covers_every_row_once():
    from gnnc.b200 import partition as P

    for n in (1, 7, 8, 1000, 2449029):
        for world in (1, 2, 3, 4, 8):
            rows = [P.row_range(n, world, r) for r in range(world)]
            assert rows[0].begin == 0 and rows[-1].end == n
            for a, b in zip(rows, rows[1:]):
                assert a.end == b.begin
            assert all(r.count <= r.rows_per_rank for r in rows)


@pytest.mark.timeout(180)
def test_two_rank_gloo_layer_matches_single_process(tmp_path):
    import torch.multiprocessing as mp

    from oracle import gnn_oracle as O

    world = 2
    mp.spawn(_rank_main, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    got = np.concatenate([np.load(tmp_path / f"rank{r}.npy") for r in range(world)])
    rowptr, col, x, W, a_s, a_d, H, C = _problem()
    h = x @ W.t()
    asrc = (h.view(-1, H, C) * a_s.view(1, H, C)).sum(-1)
    adst = (h.view(-1, H, C) * a_d.view(1, H, C)).sum(-1)
    ref = O.gat_rows_fp64(rowptr, col, h, asrc, adst, H).numpy()
    np.testing.assert_allclose(got, ref, rtol=1e-12, atol=1e-12)


def test_peer_read_order_starts_local_and_spreads_owners():
    from gnnc.b200 import partition as P

    for world in (1, 2, 4, 8):
        orders = [P.read_order(P.row_range(1000, world, r)) for r in range(world)]
        for r, order in enumerate(orders):
            assert order[0] == r and sorted(order) == list(range(world))
        # at every position k of the read sequence the ranks read distinct owners
        for k in range(world):
            assert len({o[k] for o in orders}) == world


def _rank_needed(rank, world, port, out_dir):
    sys.path[:0] = [ROOT, os.path.join(ROOT, "ml-reentry-mlir_b200")]
    import torch.distributed as dist

    from gnnc.b200 import partition as P

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world)
    rowptr, col, x, W, a_s, a_d, H, C = _problem()
    n = x.size(0)
    rr = P.row_range(n, world, rank)
    rowptr_l, col_l = P.local_csr(rowptr, col, rr)
    plan = P.NeededRows(col_l.to(torch.int32), rr)
    R = rr.rows_per_rank
    x_own = torch.zeros(R, x.size(1), dtype=x.dtype)
    x_own[: rr.count] = x[rr.begin : rr.end]
    packed = x_own[plan.pack_idx.long()]  # the owner-side pack
    blocks: list = [None] * world
    dist.all_gather_object(blocks, packed)  # stands in for the peer pulls
    table = torch.zeros(plan.compact_rows, x.size(1), dtype=x.dtype)
    table[:R] = x_own
    for p in range(world):
        if p != rank and plan.need_rows[p]:
            off = plan.remote_off[p]
            table[plan.base[p] : plan.base[p] + plan.need_rows[p]] = blocks[p][off : off + plan.need_rows[p]]
    ok = torch.equal(table[plan.col.long()], x[col_l.long()])
    # requester-side gathers: rows need_idx[p] of owner p's block land at base[p]
    owners: list = [None] * world
    dist.all_gather_object(owners, x_own)  # stands in for the mapped blocks
    table2 = torch.zeros_like(table)
    table2[:R] = x_own
    for p in range(world):
        if p != rank and plan.need_rows[p]:
            table2[plan.base[p] : plan.base[p] + plan.need_rows[p]] = owners[p][plan.need_idx[p].long()]
    ok_gather = torch.equal(table2, table)
    frac = sum(plan.need_rows) / max(1, n - rr.count)
    torch.save({"ok": ok, "ok_gather": ok_gather, "frac": frac},
               os.path.join(out_dir, f"n{rank}.pt"))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.timeout(180)
def test_needed_rows_relabel_and_offsets_gloo(tmp_path):
    """Three ranks: each packs the rows the others need, the blocks travel
    (all_gather here, peer pulls on the GPU), and the compact table indexed by
    the relabelled columns gives every edge its source row; the requester-side
    gathers (need_idx per owner) build the same table."""
    import torch.multiprocessing as mp

    world = 3
    mp.spawn(_rank_needed, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    for r in range(world):
        got = torch.load(tmp_path / f"n{r}.pt")
        assert got["ok"] and got["ok_gather"]
        assert 0.0 < got["frac"] <= 1.0


def test_whole_graph_split_threshold_formula():
    """gnnc_plan_create's default: max(4096, edges / (2 * SMs * 4)), capped at 2^30."""
    from gnnc.b200 import partition as P

    assert P.whole_graph_split_threshold(64_308_169, 148) == 64_308_169 // 1184
    assert P.whole_graph_split_threshold(1000, 148) == 4096
    assert P.whole_graph_split_threshold(1 << 45, 148) == 1 << 30


def _fence_rank(rank, world, port, out_dir):
    sys.path[:0] = [ROOT, os.path.join(ROOT, "ml-reentry-mlir_b200")]
    import time
    from datetime import timedelta

    import torch.distributed as dist

    from gnnc.b200.distributed import host_fence

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=timedelta(seconds=60))
    host_fence(timeout=timedelta(seconds=20))  # step 1: every rank arrives
    if rank == 1:
        time.sleep(12)  # stops between steps: never reaches the second fence
        return
    t0 = time.monotonic()
    try:
        host_fence(timeout=timedelta(seconds=2))
        msg = "PASSED"
    except RuntimeError as exc:
        msg = f"RAISED {exc}"
    with open(os.path.join(out_dir, "fence.txt"), "w") as f:
        f.write(f"{time.monotonic() - t0:.3f}\n{msg}\n")


def test_host_fence_names_a_rank_that_stopped_arriving(tmp_path):
    """A rank that stops between steps: the next host fence raises on rank 0
    within its 2 s bound, naming rank 1, instead of waiting out the process
    group's 60 s timeout (gloo, two processes, no GPU)."""
    import torch.multiprocessing as mp

    mp.spawn(_fence_rank, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True)
    waited, msg = (tmp_path / "fence.txt").read_text().splitlines()[:2]
    assert msg.startswith("RAISED") and "1" in msg, msg
    assert 1.5 <= float(waited) < 10.0, waited
