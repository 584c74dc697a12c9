"""1-D destination-row partitioning of one GCN / GAT layer across ranks.

The reference has no multi-GPU path (multi-GPU is deferred,
internal-docs/project-summary.md:105). Here a layer runs on `world` GPUs, one
process per GPU:

  1. rank r owns destination rows [r*R, min(N, (r+1)*R)), R = ceil(N / world),
     with its slice of the CSR (all source columns stay global);
  2. each rank projects its own rows into its R-row slot of a [world*R, F]
     table (its slot of the all-gather buffer, so no copy is needed);
  3. the table (and GAT's a_src) is all-gathered over NCCL - the path's one
     exchange step;
  4. each rank aggregates its rows from the gathered table.

Equal row counts keep the all-gather uniform; with node ids assigned
independently of degree (as in the configuration-model and R-MAT workloads)
they are also edge-balanced to about one percent.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class RowRange:
    rank: int
    world: int
    rows_per_rank: int  # R (slot height in the gathered table)
    begin: int
    end: int

    @property
    def count(self) -> int:
        return self.end - self.begin


def row_range(num_nodes: int, world: int, rank: int) -> RowRange:
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of {world}")
    R = (num_nodes + world - 1) // world
    b = min(num_nodes, rank * R)
    return RowRange(rank, world, R, b, min(num_nodes, b + R))


def local_csr(rowptr: torch.Tensor, col: torch.Tensor, rr: RowRange, extra: tuple = ()):
    """The rows [rr.begin, rr.end) of a CSR, rebased to start at edge 0.

    Returns (rowptr_local int32 [count+1], col_local, *extra_local) where each
    tensor in `extra` is an edge array (weights, scores) sliced the same way."""
    e0, e1 = (int(v) for v in rowptr[[rr.begin, rr.end]].tolist())
    rp = (rowptr[rr.begin : rr.end + 1] - e0).to(torch.int32).contiguous()
    out = [rp, col[e0:e1].contiguous()]
    out += [t[e0:e1].contiguous() for t in extra]
    return tuple(out)


def gathered_table(rr: RowRange, width: int, dtype: torch.dtype, device) -> torch.Tensor:
    """[world*R, width] all-gather buffer; rank r's slot is rows [r*R, r*R + R)."""
    return torch.empty((rr.world * rr.rows_per_rank, width), dtype=dtype, device=device)


def my_slot(table: torch.Tensor, rr: RowRange) -> torch.Tensor:
    """This rank's R-row slot of the gathered table (the all-gather input)."""
    b = rr.rank * rr.rows_per_rank
    return table[b : b + rr.rows_per_rank]


def my_rows(table: torch.Tensor, rr: RowRange) -> torch.Tensor:
    """The live rows of this rank's slot (count may be < R on the last rank)."""
    b = rr.rank * rr.rows_per_rank
    return table[b : b + rr.count]


def all_gather_rows(table: torch.Tensor, rr: RowRange, group=None) -> None:
    """In-place all-gather of every rank's slot into `table` (no-op for one rank)."""
    if rr.world == 1:
        return
    import torch.distributed as dist

    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(table, my_slot(table, rr), group=group)
    else:  # gloo (CPU tests): the list form of the same collective
        dist.all_gather(list(table.split(rr.rows_per_rank)), my_slot(table, rr).clone(), group=group)
