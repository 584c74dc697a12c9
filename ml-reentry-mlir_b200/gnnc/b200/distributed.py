"""Whole-model forward on `world` GPUs, one process per GPU.

The reference has no multi-GPU path (internal-docs/project-summary.md:105).
Here a lowered model (B200Executable) runs its layers partitioned by
destination row: rank r owns rows [r*R, (r+1)*R), R = ceil(N / world), their
input features and their output rows. Each layer has one exchange step, over
the narrower side of its projection:

* input exchange (the layer's input is narrower than its projected rows, e.g.
  100 -> 4 x 64): every rank keeps its input rows in its slot of a
  [world*R, K] table; the copy engines pull the other slots from the owners'
  HBM (CUDA IPC mapping, gnnc_peer_copy) piece by piece while the projection
  runs on the pieces already present, so every rank projects all rows;
* output exchange (the projected rows are narrower, e.g. 256 -> 47): each rank
  projects its own rows into its slot of the [world*R, F] table (and a_src's
  for GAT), and the other slots are pulled the same way.

The layer's aggregation then reads local memory only and writes its rows
straight into the next layer's input slot. For a stream of batches,
run_stream pipelines the first layer's input exchange across them: batch
k+1's rows are pulled into a second table while batch k aggregates. A fence orders each exchanged
buffer's writes before the peers' reads (a one-word NCCL all-reduce on the
stream, or a host barrier for gloo process groups that names a rank which
stopped arriving, `host_fence`), and one more at the end of
the forward orders the last reads before the next forward's writes. The
results are those of the single-GPU executable, row for row: every row is
projected and aggregated by the same kernels on the same values.
"""

from __future__ import annotations

from dataclasses import dataclass
from datetime import timedelta

import torch

from gnnc.b200 import partition as P
from gnnc.b200 import runtime as rt
from gnnc.b200.program import B200Executable


def host_fence(group=None, timeout: timedelta = timedelta(seconds=60)) -> None:
    """Host barrier over a gloo group that detects a rank that is gone.

    torch.distributed.monitored_barrier: rank 0 waits for every other rank up
    to `timeout`; a rank that died or stopped between steps makes the barrier
    raise RuntimeError naming it (on rank 0; the others see their barrier
    fail), instead of every rank waiting out the process group's own timeout."""
    import torch.distributed as dist

    dist.monitored_barrier(group=group, timeout=timeout, wait_all_ranks=True)


@dataclass
class _Layer:
    mode: str  # "input" | "output"
    rowptr: torch.Tensor
    col: torch.Tensor
    w: torch.Tensor | None
    plan: rt.Plan
    table: torch.Tensor  # exchanged [world*R, ld] (input rows or projected rows)
    peers: _PeerTable
    in_own: torch.Tensor  # this rank's input rows [R, ld_in] (a view of table for input mode)
    h_full: torch.Tensor  # projected rows of every node [world*R, F]
    a_full: torch.Tensor | None  # GAT a_src [world*R, H] (exchanged in output mode)
    a_peers: _PeerTable | None
    d_full: torch.Tensor | None  # GAT a_dst [world*R, H] (own rows used)
    root: torch.Tensor | None  # SAGE lin_r rows of this rank [R, F]


class _PeerTable:
    """Every rank's copy of one [world*R, ld] table, mapped into this process;
    slot(p, a, b) addresses rows [a, b) of rank p's own slot in rank p's table."""

    def __init__(self, table: torch.Tensor, rr: P.RowRange, group) -> None:
        import torch.distributed as dist

        self.table, self.rr = table, rr
        meta: list = [None] * rr.world
        dist.all_gather_object(meta, rt.peer_export(table), group=group)
        self.ptrs: list[int] = []
        self._opened: list[tuple[int, int]] = []
        for p in range(rr.world):
            if p == rr.rank:
                self.ptrs.append(table.data_ptr())
            else:
                handle, off = meta[p]
                ptr = rt.peer_open(table.device, handle, off)
                self._opened.append((ptr, off))
                self.ptrs.append(ptr)

    def slot(self, p: int, a: int, b: int) -> rt.DeviceRows:
        t = self.table
        row_bytes = t.stride(0) * t.element_size()
        base = self.ptrs[p] + (p * self.rr.rows_per_rank + a) * row_bytes
        return rt.DeviceRows(base, b - a, t.size(1), t.stride(0), t.dtype, t.device)

    def close(self) -> None:
        for ptr, off in self._opened:
            rt.peer_close(self.table.device, ptr, off)
        self._opened = []


class DistributedExecutable:
    """A B200Executable run partitioned over the ranks of `group`.

    Call with (x_rows, graph): x_rows are this rank's input rows
    [rows of row_range(N, world, rank)], graph the whole graph (the adjacency
    or edge_index every rank holds). Returns this rank's output rows."""

    PIECE_ROWS = 1 << 18

    def __init__(self, exe: B200Executable, group=None, fence: str = "auto",
                 fence_timeout: timedelta = timedelta(seconds=60)) -> None:
        import torch.distributed as dist

        self.exe, self.program, self.device = exe, exe.program, exe.device
        self.group = group
        self.fence_timeout = fence_timeout
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if fence == "auto":
            fence = "nccl" if dist.get_backend(group) == "nccl" else "host"
        if fence not in ("nccl", "host"):
            raise ValueError(f"unknown fence {fence!r}")
        self.fence_kind = fence
        self._fence_buf = torch.zeros(1, dtype=torch.int32, device=self.device)
        self._side = torch.cuda.Stream(self.device)
        self._key = None
        self._layers: list[_Layer] = []
        self._out: torch.Tensor | None = None
        self._rr: P.RowRange | None = None
        self._second: tuple[torch.Tensor, _PeerTable] | None = None  # run_stream's 2nd table

    # -- set-up ------------------------------------------------------------

    def _fence(self) -> None:
        import torch.distributed as dist

        if self.fence_kind == "nccl":
            dist.all_reduce(self._fence_buf, group=self.group)
        else:
            torch.cuda.synchronize(self.device)
            host_fence(self.group, self.fence_timeout)

    def exchange_modes(self) -> list[str]:
        """Per layer, the side of the projection that crosses NVLink."""
        s = torch.empty((), dtype=self.program.feature_dtype).element_size()
        modes = []
        for layer in self.program.layers:
            in_b = rt.row_stride(layer.in_channels, self.program.feature_dtype) * s
            out_b = rt.row_stride(layer.width, self.program.feature_dtype) * s
            if layer.kind == "gat":
                out_b += 4 * layer.heads
            modes.append("input" if in_b <= out_b else "output")
        return modes

    def _setup(self, x_rows: torch.Tensor, graph: torch.Tensor) -> None:
        import torch.distributed as dist

        counts: list = [None] * self.world
        dist.all_gather_object(counts, int(x_rows.size(0)), group=self.group)
        N = int(sum(counts))
        rr = P.row_range(N, self.world, self.rank)
        if [P.row_range(N, self.world, r).count for r in range(self.world)] != counts:
            raise ValueError(f"ranks hold {counts} rows; row_range({N}, {self.world}) expects "
                             "equal contiguous ranges")
        self.close()
        self._rr, R, W = rr, rr.rows_per_rank, self.world
        self._key = (None, N)
        dev, dt = self.device, self.program.feature_dtype
        layers = []
        modes = self.exchange_modes()
        for layer, mode in zip(self.program.layers, modes, strict=True):
            g = self.exe._graph_for(graph, N, layer)
            extra = () if g.w is None else (g.w,)
            parts = P.local_csr(g.rowptr, g.col, rr, extra)
            rowptr_l, col_l = parts[0], parts[1]
            w_l = parts[2] if g.w is not None else None
            # the single-GPU plan's split decisions (bit-identical rows)
            sms = torch.cuda.get_device_properties(dev).multi_processor_count
            plan = rt.Plan(rowptr_l, split_threshold=P.whole_graph_split_threshold(
                g.col.numel(), sms))
            ld_in = rt.row_stride(layer.in_channels, dt)
            ld_f = rt.row_stride(layer.width, dt)
            gat = layer.kind == "gat"
            H = layer.heads
            h_full = torch.zeros((W * R, ld_f), dtype=dt, device=dev)
            a_full = torch.zeros((W * R, H), dtype=torch.float32, device=dev) if gat else None
            d_full = torch.zeros((W * R, H), dtype=torch.float32, device=dev) if gat else None
            if mode == "input":
                table = torch.zeros((W * R, ld_in), dtype=dt, device=dev)
                in_own = table[rr.begin : rr.begin + R]
                peers, a_peers = _PeerTable(table, rr, self.group), None
            else:
                table = h_full
                in_own = torch.zeros((R, ld_in), dtype=dt, device=dev)
                peers = _PeerTable(table, rr, self.group)
                a_peers = _PeerTable(a_full, rr, self.group) if gat else None
            root = (torch.zeros((R, ld_f), dtype=dt, device=dev)
                    if layer.kind == "sage" else None)
            layers.append(_Layer(mode, rowptr_l, col_l, w_l, plan, table, peers, in_own, h_full,
                                 a_full, a_peers, d_full, root))
        last = self.program.layers[-1]
        self._out = rt.empty_rows(R, last.out_width, self.program.output_dtype, dev)
        self._layers = layers
        self._key = (self.exe._graph_key(graph), N)

    def close(self) -> None:
        """Unmaps the peers' tables (collective: every rank calls it)."""
        for L in self._layers:
            L.peers.close()
            if L.a_peers is not None:
                L.a_peers.close()
        if self._second is not None:
            self._second[1].close()
            self._second = None
        self._layers = []
        self._key = None

    # -- forward -----------------------------------------------------------

    def _pull(self, table: _PeerTable, dst: torch.Tensor, events: list) -> None:
        """Copies every other rank's slot of `table` into the same rows of
        `dst`, in pieces on the side stream; appends (row slice, event) per
        piece to `events`. Owners are read in rotated order (rank r reads r+1,
        r+2, ...), so at any time each owner serves one reader."""
        rr, R, N = self._rr, self._rr.rows_per_rank, self._key[1]
        row_bytes = dst.stride(0) * dst.element_size()
        for k in range(1, self.world):
            p = (rr.rank + k) % self.world
            n_p = P.row_range(N, rr.world, p).count
            for a in range(0, n_p, self.PIECE_ROWS):
                b = min(n_p, a + self.PIECE_ROWS)
                rt.peer_copy(dst[p * R + a :], table.slot(p, a, b), (b - a) * row_bytes)
                ev = torch.cuda.Event()
                ev.record(self._side)
                events.append((slice(p * R + a, p * R + b), ev))

    def run_device(self, x_rows: torch.Tensor, graph: torch.Tensor) -> torch.Tensor:
        """Forward of this rank's rows; returns them on the device. Collective:
        every rank of the group calls it with the same graph."""
        if self._key is None or self._key[0] != self.exe._graph_key(graph):
            self._setup(x_rows, graph)
        n = self._rr.count
        with torch.cuda.device(self.device):
            first = self._layers[0]
            first.in_own[:n, : self.program.layers[0].in_channels].copy_(x_rows, non_blocking=True)
            for i in range(len(self._layers)):
                self._layer(i)
            self._fence()  # every peer is done reading this forward's rows
        return self._out[:n]

    def run_stream(self, batches, graph: torch.Tensor):
        """Forwards of a stream of batches, pipelined across them.

        `batches` yields this rank's input rows of each batch (host or device
        tensors, the rows run_device takes). When the first layer exchanges its
        input rows, the copy engines pull batch k+1's remote input rows while
        batch k aggregates (two input tables, each mapped by the peers), so that
        exchange leaves the critical path; the other layers run as in
        run_device. Yields this rank's output rows of each batch on the device,
        valid until the next batch is requested; each equals run_device's
        result for that batch. Collective: every rank iterates the same number
        of batches with the same graph."""
        it = iter(batches)
        x = next(it, None)
        if x is None:
            return
        if self._key is None or self._key[0] != self.exe._graph_key(graph):
            self._setup(x, graph)
        if self.world == 1 or self._layers[0].mode != "input":
            while x is not None:
                yield self.run_device(x, graph)
                x = next(it, None)
            return
        rr, N = self._rr, self._key[1]
        n, K0 = rr.count, self.program.layers[0].in_channels
        L0 = self._layers[0]
        if self._second is None:
            t = torch.zeros_like(L0.table)
            self._second = (t, _PeerTable(t, rr, self.group))
        tabs = (L0.table, self._second[0])
        peers = (L0.peers, self._second[1])
        cur = torch.cuda.current_stream(self.device)
        pulled = (torch.cuda.Event(), torch.cuda.Event())

        def pull(b: int) -> None:
            self._side.wait_stream(cur)
            with torch.cuda.stream(self._side):
                self._pull(peers[b], tabs[b], [])
                pulled[b].record(self._side)

        with torch.cuda.device(self.device):
            tabs[0][rr.begin : rr.begin + n, :K0].copy_(x, non_blocking=True)
            self._fence()  # batch 0's input rows are written on every rank
            pull(0)
            k = 0
            while x is not None:
                nxt = next(it, None)
                b = k % 2
                cur.wait_event(pulled[b])  # batch k's remote rows are present
                if nxt is not None:
                    # this slot's previous batch (k-1) was pulled before the last fence
                    tabs[1 - b][rr.begin : rr.begin + n, :K0].copy_(nxt, non_blocking=True)
                # every rank holds batch k's rows and wrote batch k+1's own rows
                self._fence()
                self._layer(0, table=tabs[b][:N], pull_next=(lambda: pull(1 - b))
                            if nxt is not None else None)
                for i in range(1, len(self._layers)):
                    self._layer(i)
                self._fence()  # every peer is done reading this batch's rows
                yield self._out[:n]
                x, k = nxt, k + 1

    def _layer(self, i: int, table: torch.Tensor | None = None, pull_next=None) -> None:
        """Layer i of a forward on the current stream: its exchange, projection
        and aggregation into the next layer's input slot (or the output).
        `table` is the first layer's input table with every rank's rows already
        present (a batch of run_stream): it is projected in one launch, and
        `pull_next` then starts the next batch's pull before the aggregation."""
        rr, layer, L = self._rr, self.program.layers[i], self._layers[i]
        w, asw, adw, bias = self.exe._weights[i]
        wr = self.exe._roots[i]
        n, dt = rr.count, self.program.feature_dtype
        cur = torch.cuda.current_stream(self.device)
        K, F = layer.in_channels, layer.width
        gat = layer.kind == "gat"

        def proj(x, rows: slice):
            if gat:
                rt.proj(x, w, att_src=asw, att_dst=adw, heads=layer.heads, out_dtype=dt,
                        out=L.h_full[rows, :F], asrc_out=L.a_full[rows], adst_out=L.d_full[rows])
            else:
                rt.proj(x, w, out_dtype=dt, out=L.h_full[rows, :F])

        own = slice(rr.begin, rr.begin + n)
        x_own = L.in_own
        events: list = []
        if table is not None:
            proj(table[:, :K], slice(0, table.size(0)))
            x_own = table[rr.begin : rr.begin + rr.rows_per_rank]
        elif L.mode == "input":
            self._fence()  # this layer's input rows are written on every rank
            self._side.wait_stream(cur)
            with torch.cuda.stream(self._side):
                self._pull(L.peers, L.table, events)
            if n:
                proj(L.in_own[:n, :K], own)
            for rows, ev in events:
                cur.wait_event(ev)
                proj(L.table[rows, :K], rows)
        else:
            if n:
                proj(L.in_own[:n, :K], own)
            self._fence()  # projected rows written everywhere
            self._side.wait_stream(cur)
            with torch.cuda.stream(self._side):
                self._pull(L.peers, L.h_full, events)
                if gat:
                    self._pull(L.a_peers, L.a_full, events)
            for _, ev in events:
                cur.wait_event(ev)
        if layer.kind == "sage" and n:
            rt.proj(x_own[:n, :K], wr, out_dtype=dt, out=L.root[:n, :F])
        if pull_next is not None:
            pull_next()
        if i == len(self._layers) - 1:
            out = self._out[:n]
        else:
            out = self._layers[i + 1].in_own[:n, : self.program.layers[i + 1].in_channels]
        if n:
            self._aggregate(layer, L, n, bias, out)

    def _aggregate(self, layer, L: _Layer, n: int, bias, out: torch.Tensor) -> None:
        N, F = self._key[1], layer.width
        rr = self._rr
        h = L.h_full[:N, :F]
        if layer.kind == "gat":
            rt.gat_aggregate(L.plan, L.rowptr, L.col, h, L.a_full[:N],
                             L.d_full[rr.begin : rr.begin + n], heads=layer.heads,
                             negative_slope=layer.negative_slope, concat=layer.concat,
                             bias=bias, act=layer.act, log_softmax=layer.log_softmax,
                             out_dtype=out.dtype, out=out)
        elif layer.kind == "sage":
            rt.sage_aggregate(L.plan, L.rowptr, L.col, L.w, h, L.root[:n, :F], bias=bias,
                              act=layer.act, log_softmax=layer.log_softmax, out_dtype=out.dtype,
                              out=out)
        else:
            rt.gcn_aggregate(L.plan, L.rowptr, L.col, L.w, h, bias=bias, act=layer.act,
                             log_softmax=layer.log_softmax, out_dtype=out.dtype, out=out)

    def __call__(self, x_rows: torch.Tensor, graph: torch.Tensor) -> torch.Tensor:
        out = self.run_device(x_rows, graph)
        if not x_rows.is_cuda:
            host = torch.empty(tuple(out.shape), dtype=out.dtype, pin_memory=True)
            host.copy_(out, non_blocking=True)
            torch.cuda.current_stream(self.device).synchronize()
            return host
        return out.contiguous()


def distribute(exe: B200Executable, group=None, fence: str = "auto",
               fence_timeout: timedelta = timedelta(seconds=60)) -> DistributedExecutable:
    """Wraps a compiled executable for a row-partitioned forward over `group`."""
    if not isinstance(exe, B200Executable):
        raise NotImplementedError(f"cannot distribute {type(exe).__name__}")
    return DistributedExecutable(exe, group=group, fence=fence, fence_timeout=fence_timeout)


__all__ = ["DistributedExecutable", "distribute", "host_fence"]
