"""1-D destination-row partitioning of one GCN / GAT layer across ranks.

The reference has no multi-GPU path (multi-GPU is deferred,
internal-docs/project-summary.md:105). Here a layer runs on `world` GPUs, one
process per GPU, each owning a set of destination rows with its slice of the
CSR (all source columns stay global). The layer's one exchange step is an
all-gather over NCCL of one side of the projection, whichever is narrower:

* output exchange (`RowRange`): rank r owns rows [r*R, min(N, (r+1)*R)),
  R = ceil(N / world); it projects its own rows into its R-row slot of a
  [world*R, F] table (its slot of the all-gather buffer, so no copy is
  needed), the table (and GAT's a_src) is all-gathered, and each rank
  aggregates its rows. Bytes exchanged per row: F (+ H for GAT) values.

* peer reads (`PeerRows`): rank r owns rows [r*R, (r+1)*R) and their input
  rows; every rank maps every other rank's input buffer (CUDA IPC) and its
  projection reads the remote rows over NVLink inside its own tile loads,
  writing h for all rows locally. No collective moves data; two one-word
  all-reduces per layer order the buffer's writes and the peers' reads.
  Bytes over NVLink per row: K input values, as for the input exchange, but
  without a separate copy pass.

* input exchange (`RowBlocks`): the input features X are all-gathered and
  every rank projects all N rows itself. Bytes per row: K input values, so
  this wins when K < F + H (a 100-wide input projected to 4 heads x 64 moves
  208 instead of 528 bytes a row). The gather is split into `chunks` pieces so
  that the projection of one piece overlaps the transfer of the next; for each
  piece to land as a contiguous run of table rows in node order, ownership is
  block-cyclic: the rows, padded to chunks*world*S, form `chunks` pieces of
  world*S rows and rank r owns the r-th S-row block of every piece.

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


def whole_graph_split_threshold(total_edges: int, num_sms: int) -> int:
    """The split threshold gnnc_plan_create picks by default for a CSR of
    `total_edges` edges on a GPU of `num_sms` SMs: max(4096, edges / (2 * SMs * 4)).

    A rank's plan covers only its rows, so its own default would follow its
    smaller edge count and split rows the single-GPU plan keeps whole (a split
    row sums its edges in segments: the same value up to rounding). Giving each
    rank this threshold makes it split exactly the rows one GPU would, so the
    partitioned results equal the single-GPU results bit for bit."""
    per = int(total_edges) // (2 * int(num_sms) * 4)
    return int(min(max(4096, per), 1 << 30))


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


# ---------------------------------------------------------------------------
# input exchange: block-cyclic ownership
# ---------------------------------------------------------------------------


@dataclass(frozen=True)
class RowBlocks:
    rank: int
    world: int
    chunks: int
    block_rows: int  # S: rows per (piece, rank) block
    num_nodes: int

    @property
    def piece_rows(self) -> int:
        return self.world * self.block_rows

    @property
    def padded_rows(self) -> int:
        return self.chunks * self.piece_rows

    def piece(self, c: int) -> slice:
        """Table rows of piece c (node ids, padded past num_nodes)."""
        return slice(c * self.piece_rows, (c + 1) * self.piece_rows)

    def block(self, c: int) -> tuple[int, int]:
        """Node range [begin, end) this rank owns in piece c (clipped to num_nodes)."""
        b = c * self.piece_rows + self.rank * self.block_rows
        return min(b, self.num_nodes), min(b + self.block_rows, self.num_nodes)

    @property
    def count(self) -> int:
        """Owned rows; they are the first `count` rows of the local order
        (block 0, block 1, ...), since a clipped block is followed only by
        empty ones."""
        return sum(e - b for b, e in (self.block(c) for c in range(self.chunks)))

    def node_ids(self) -> torch.Tensor:
        """Node id of every owned row, in local order."""
        return torch.cat([torch.arange(*self.block(c), dtype=torch.int64) for c in range(self.chunks)])


def row_blocks(num_nodes: int, world: int, rank: int, chunks: int = 1) -> RowBlocks:
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of {world}")
    if chunks < 1:
        raise ValueError("chunks must be >= 1")
    S = max(1, (num_nodes + chunks * world - 1) // (chunks * world))
    return RowBlocks(rank, world, chunks, S, num_nodes)


def local_csr_blocks(rowptr: torch.Tensor, col: torch.Tensor, rb: RowBlocks, extra: tuple = ()):
    """The owned rows of a CSR, in local order, rebased to start at edge 0.

    Returns (rowptr_local int32 [count+1], col_local, *extra_local)."""
    bounds = [rb.block(c) for c in range(rb.chunks)]
    bounds = [(b, e) for b, e in bounds if e > b]
    ptrs, cols, extras = [], [], [[] for _ in extra]
    base = 0
    for b, e in bounds:
        e0, e1 = (int(v) for v in rowptr[[b, e]].tolist())
        ptrs.append(rowptr[b:e] - e0 + base)
        cols.append(col[e0:e1])
        for lst, t in zip(extras, extra):
            lst.append(t[e0:e1])
        base += e1 - e0
    end = torch.tensor([base], dtype=rowptr.dtype, device=rowptr.device)
    rp = torch.cat(ptrs + [end]).to(torch.int32).contiguous()
    out = [rp, torch.cat(cols).contiguous() if cols else col[:0].clone()]
    out += [torch.cat(lst).contiguous() if lst else t[:0].clone() for lst, t in zip(extras, extra)]
    return tuple(out)


def input_table(rb: RowBlocks, width: int, dtype: torch.dtype, device) -> torch.Tensor:
    """[padded_rows, width] table of the gathered input, in node order."""
    return torch.empty((rb.padded_rows, width), dtype=dtype, device=device)


def local_blocks(rb: RowBlocks, width: int, dtype: torch.dtype, device) -> torch.Tensor:
    """[chunks*S, width] buffer of this rank's own rows (block c = rows [c*S, (c+1)*S))."""
    return torch.zeros((rb.chunks * rb.block_rows, width), dtype=dtype, device=device)


def gather_piece(table: torch.Tensor, local: torch.Tensor, rb: RowBlocks, c: int, group=None) -> None:
    """All-gather piece c: every rank's block c of `local` lands in table[piece(c)].

    With one rank it is a copy (no-op when `local` already is the table)."""
    dst = table[rb.piece(c)]
    src = local[c * rb.block_rows : (c + 1) * rb.block_rows]
    if rb.world == 1:
        if dst.data_ptr() != src.data_ptr():
            dst.copy_(src)
        return
    import torch.distributed as dist

    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(dst, src, group=group)
    else:  # gloo (CPU tests): the list form of the same collective
        dist.all_gather(list(dst.split(rb.block_rows)), src.clone(), group=group)


def owned_rows(table: torch.Tensor, rb: RowBlocks) -> torch.Tensor:
    """Copy of this rank's rows of a [padded_rows, W] node-order table, in local order."""
    W = table.size(1)
    v = table.view(rb.chunks, rb.world, rb.block_rows, W)[:, rb.rank]
    return v.reshape(rb.chunks * rb.block_rows, W)[: rb.count]


# ---------------------------------------------------------------------------
# peer reads: every rank's input rows mapped into this process
# ---------------------------------------------------------------------------


class PeerRows:
    """Every rank's [R, ld] input row block, addressable from this rank.

    `local` is this rank's block (rows beyond its count are padding). Each rank
    exports its block's CUDA IPC handle, the handles are all-gathered (host
    objects over the process group), and the other ranks' blocks are mapped.
    view(p) is rank p's live rows as a runtime.DeviceRows (this rank's own
    block is read in place)."""

    def __init__(self, local: torch.Tensor, rr: RowRange, num_nodes: int, group=None) -> None:
        from gnnc.b200 import runtime as rt

        if local.dim() != 2 or not local.is_contiguous() or local.size(0) != rr.rows_per_rank:
            raise ValueError("local must be a contiguous [rows_per_rank, ld] block")
        self._rt = rt
        self.rr, self.local, self.num_nodes = rr, local, num_nodes
        self._opened: list[tuple[int, int]] = []
        meta: list = [None] * rr.world
        if rr.world > 1:
            import torch.distributed as dist

            dist.all_gather_object(meta, rt.peer_export(local), group=group)
        self.ptrs: list[int] = []
        for p in range(rr.world):
            if p == rr.rank:
                self.ptrs.append(local.data_ptr())
            else:
                handle, off = meta[p]
                ptr = rt.peer_open(local.device, handle, off)
                self._opened.append((ptr, off))
                self.ptrs.append(ptr)

    def view(self, p: int, cols: int):
        """Rank p's live rows [count_p, cols] (row stride = the block's ld)."""
        loc = self.local
        n = row_range(self.num_nodes, self.rr.world, p).count
        return self._rt.DeviceRows(self.ptrs[p], n, cols, loc.size(1), loc.dtype, loc.device)

    def close(self) -> None:
        for ptr, off in self._opened:
            self._rt.peer_close(self.local.device, ptr, off)
        self._opened = []


def read_order(rr: RowRange) -> list[int]:
    """Owners in the order a rank reads them: itself first, then the next
    ranks cyclically, so that at any moment the ranks read different peers."""
    return [(rr.rank + k) % rr.world for k in range(rr.world)]


# ---------------------------------------------------------------------------
# needed rows: only the remote rows a rank's edges read cross NVLink
# ---------------------------------------------------------------------------


class NeededRows:
    """Which remote input rows a rank's edges read, and how they travel.

    With contiguous row ranges, rank r's edges read the rows of every other
    rank p, but on a power-law graph only a part of them (about two thirds of
    the remote rows at 8 ranks on the 2.45M-node configuration-model graph).
    need[p] lists them (sorted offsets into p's rows). The ranks swap these
    lists once; then, per forward:

    * as owner, a rank packs for each requester q the rows q needs into one
      contiguous block of its pack buffer (`pack_idx`, block q at
      `pack_off[q]`), so a requester pulls one block per owner;
    * as requester, a rank lands owner p's block at rows `base[p]` of its
      compact table, whose first R rows are its own;
    * `col` is the local CSR's column array relabelled to compact-table rows.

    `need_idx[p]` keeps the requester's list for owner p on the device, for a
    requester that gathers the rows itself from p's mapped block (no pack).
    """

    def __init__(self, col_l: torch.Tensor, rr: RowRange, group=None) -> None:
        import torch.distributed as dist

        R, W, me = rr.rows_per_rank, rr.world, rr.rank
        dev = col_l.device
        c = col_l.long()
        uniq = torch.unique(c)
        owner = uniq // R
        need = [(uniq[owner == p] - p * R).to(torch.int32) for p in range(W)]
        need[me] = need[me][:0]
        lists: list = [None] * W
        dist.all_gather_object(lists, [t.cpu() for t in need], group=group)
        send = [lists[q][me] if q != me else torch.empty(0, dtype=torch.int32) for q in range(W)]
        sizes = [int(t.numel()) for t in send]
        self.pack_off = [sum(sizes[:q]) for q in range(W)]
        self.pack_rows = sum(sizes)
        self.pack_idx = (torch.cat(send).to(dev) if self.pack_rows
                         else torch.empty(0, dtype=torch.int32, device=dev))
        offs: list = [None] * W
        dist.all_gather_object(offs, self.pack_off, group=group)
        self.remote_off = [offs[p][me] for p in range(W)]  # my block in p's pack buffer
        self.need_rows = [int(t.numel()) for t in need]
        self.need_idx = [t.to(dev) for t in need]
        self.base = [0] * W
        nxt = R
        for p in read_order(rr)[1:]:
            self.base[p] = nxt
            nxt += self.need_rows[p]
        self.compact_rows = nxt
        comp = torch.empty_like(c)
        src_owner = c // R
        mine = src_owner == me
        comp[mine] = c[mine] - me * R
        for p in range(W):
            if p == me or not self.need_rows[p]:
                continue
            m = src_owner == p
            comp[m] = self.base[p] + torch.searchsorted(need[p].long(), c[m] - p * R)
        self.col = comp.to(torch.int32).contiguous()
        self.rr = rr


class PeerBuffers:
    """Every rank's copy of a row buffer (rows may differ per rank, the row
    stride may not), mapped into this process over CUDA IPC; rows(p, a, b)
    addresses rows [a, b) of rank p's buffer."""

    def __init__(self, local: torch.Tensor, group=None) -> None:
        import torch.distributed as dist

        from gnnc.b200 import runtime as rt

        self._rt, self.local = rt, local
        world, me = dist.get_world_size(group), dist.get_rank(group)
        meta: list = [None] * world
        dist.all_gather_object(meta, rt.peer_export(local), group=group)
        self.ptrs: list[int] = []
        self._opened: list[tuple[int, int]] = []
        for p in range(world):
            if p == me:
                self.ptrs.append(local.data_ptr())
            else:
                handle, off = meta[p]
                ptr = rt.peer_open(local.device, handle, off)
                self._opened.append((ptr, off))
                self.ptrs.append(ptr)

    def rows(self, p: int, a: int, b: int):
        t = self.local
        rb = t.stride(0) * t.element_size()
        return self._rt.DeviceRows(self.ptrs[p] + a * rb, b - a, t.size(1), t.stride(0), t.dtype,
                                   t.device)

    def close(self) -> None:
        for ptr, off in self._opened:
            self._rt.peer_close(self.local.device, ptr, off)
        self._opened = []
