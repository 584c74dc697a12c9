"""B200 lowering: torch model -> kernel program -> executable.

The reference lowers a PyG model through torch.export, torch-mlir and the MLIR
sparsifier (gnnc/compile.py:109-124, gnnc/schedule/sparse.py:21-114); its
aggregation reaches the backend as aten._sparse_mm (test/reference/gcn.raw.mlir:7).
The B200 target instead traces the model with torch.fx, keeping GCNConv /
GATConv / SAGEConv modules as leaves, and matches the chain

    x -> conv -> [relu | elu] -> [dropout(eval)] -> conv -> ... -> [log_softmax]

into one LayerOp per conv. Each LayerOp becomes two kernel launches: the dense
projection (gnnc_proj, with GAT's attention coefficients in its epilogue) and
the aggregation (gnnc_gcn_aggregate / gnnc_gat_aggregate) with bias, the
activation and the final log_softmax fused into its epilogue. A SAGEConv layer
projects twice (lin_l for the neighbours, lin_r for the root) and aggregates
with gnnc_sage_aggregate on mean-normalised edge weights (the reference's
`_sparse_mm.reduce("mean")`, test/reference/sage.raw.mlir:5), adding the root
term in the epilogue.
"""

from __future__ import annotations

import operator
import sys
from dataclasses import dataclass, field

import torch
import torch.fx as fx
import torch.nn.functional as F

from gnnc.b200 import runtime as rt

_CONV_CLASSES = ("GCNConv", "GATConv", "SAGEConv")


def _is_conv(mod: torch.nn.Module) -> bool:
    return type(mod).__name__ in _CONV_CLASSES


class _Tracer(fx.Tracer):
    def is_leaf_module(self, m: torch.nn.Module, qualname: str) -> bool:
        return _is_conv(m) or super().is_leaf_module(m, qualname)


def trace(model: torch.nn.Module) -> fx.GraphModule:
    """fx graph of `model` with GCNConv / GATConv / SAGEConv kept as call_module leaves."""
    model.eval()
    graph = _Tracer().trace(model)
    return fx.GraphModule(model, graph)


@dataclass
class LayerOp:
    name: str
    kind: str  # "gcn" | "gat"
    in_channels: int
    heads: int
    channels: int  # per head
    concat: bool
    negative_slope: float
    normalize: bool
    add_self_loops: bool
    weight: torch.Tensor  # [heads*channels, in]
    att_src: torch.Tensor | None
    att_dst: torch.Tensor | None
    bias: torch.Tensor | None
    act: int = rt.ACT_NONE
    log_softmax: bool = False
    weight_root: torch.Tensor | None = None  # SAGE lin_r [F, in]

    @property
    def width(self) -> int:
        return self.heads * self.channels

    @property
    def out_width(self) -> int:
        return self.width if self.concat else self.channels

    def describe(self) -> str:
        act = {rt.ACT_NONE: "none", rt.ACT_RELU: "relu", rt.ACT_ELU: "elu"}[self.act]
        proj = f"gnnc_proj [{self.in_channels} -> {self.width}]"
        if self.kind == "gat":
            proj += f" + attention coefficients (heads={self.heads})"
            agg = (
                f"gnnc_gat_aggregate heads={self.heads} C={self.channels} "
                f"slope={self.negative_slope} concat={int(self.concat)}"
            )
        elif self.kind == "sage":
            proj = (f"gnnc_proj [{self.in_channels} -> {self.width}] (lin_l) and "
                    f"[{self.in_channels} -> {self.width}] (lin_r, root)")
            agg = f"gnnc_sage_aggregate F={self.width} mean weights (gnnc_mean_norm) + root"
        else:
            agg = f"gnnc_gcn_aggregate F={self.width} normalize={int(self.normalize)}"
        epi = f"bias={'yes' if self.bias is not None else 'no'} act={act}"
        epi += " log_softmax" if self.log_softmax else ""
        return f"  {self.name}: {proj}\n  {self.name}: {agg} epilogue({epi})"


@dataclass
class B200Program:
    layers: list[LayerOp]
    input_names: list[str]
    feature_dtype: torch.dtype = torch.float32
    output_dtype: torch.dtype = torch.float32
    notes: list[str] = field(default_factory=list)

    def __str__(self) -> str:
        lines = [f"b200.program(inputs={self.input_names}, features={self.feature_dtype}, "
                 f"output={self.output_dtype})"]
        lines += [layer.describe() for layer in self.layers]
        return "\n".join(lines)


def _layer_from_module(name: str, mod: torch.nn.Module) -> LayerOp:
    cls = type(mod).__name__
    if cls == "GCNConv":
        if getattr(mod, "improved", False):
            raise NotImplementedError(f"{name}: GCNConv(improved=True) is not supported")
        lin = mod.lin
        w = lin.weight.detach()
        return LayerOp(
            name=name, kind="gcn", in_channels=w.size(1), heads=1, channels=w.size(0),
            concat=True, negative_slope=0.0, normalize=bool(getattr(mod, "normalize", True)),
            add_self_loops=bool(getattr(mod, "add_self_loops", True)), weight=w,
            att_src=None, att_dst=None,
            bias=None if mod.bias is None else mod.bias.detach(),
        )
    if cls == "SAGEConv":
        aggr = getattr(mod, "aggr", "mean")
        if str(aggr).lower() not in ("mean", "meanaggregation()"):
            raise NotImplementedError(f"{name}: SAGEConv(aggr={aggr!r}) is not supported (mean only)")
        if getattr(mod, "normalize", False) or getattr(mod, "project", False):
            raise NotImplementedError(f"{name}: SAGEConv(normalize/project) is not supported")
        if not getattr(mod, "root_weight", True):
            raise NotImplementedError(f"{name}: SAGEConv(root_weight=False) is not supported")
        wl = mod.lin_l.weight.detach()
        return LayerOp(
            name=name, kind="sage", in_channels=wl.size(1), heads=1, channels=wl.size(0),
            concat=True, negative_slope=0.0, normalize=False, add_self_loops=False, weight=wl,
            att_src=None, att_dst=None,
            bias=None if mod.lin_l.bias is None else mod.lin_l.bias.detach(),
            weight_root=mod.lin_r.weight.detach(),
        )
    # GATConv: PyG >= 2.5 names the shared projection `lin`; older releases `lin_src`.
    lin = getattr(mod, "lin", None)
    if lin is None:
        lin = mod.lin_src
        if getattr(mod, "lin_dst", lin) is not lin:
            raise NotImplementedError(f"{name}: bipartite GATConv is not supported")
    if getattr(mod, "edge_dim", None) is not None or getattr(mod, "residual", False):
        raise NotImplementedError(f"{name}: edge features / residual GATConv not supported")
    H, C = int(mod.heads), int(mod.out_channels)
    w = lin.weight.detach()
    return LayerOp(
        name=name, kind="gat", in_channels=w.size(1), heads=H, channels=C,
        concat=bool(mod.concat), negative_slope=float(mod.negative_slope), normalize=False,
        add_self_loops=bool(mod.add_self_loops), weight=w,
        att_src=mod.att_src.detach().reshape(-1), att_dst=mod.att_dst.detach().reshape(-1),
        bias=None if mod.bias is None else mod.bias.detach(),
    )


_RELU = {F.relu, torch.relu, torch.nn.functional.relu}
_ELU = {F.elu, torch.nn.functional.elu}
_LOGSM = {F.log_softmax, torch.log_softmax}
_DROPOUT = {F.dropout, torch.nn.functional.dropout}


def lower_graph(gm: fx.GraphModule, feature_dtype: torch.dtype | None = None,
                output_dtype: torch.dtype | None = None) -> B200Program:
    """Matches the conv / activation chain of `gm` into a B200Program."""
    modules = dict(gm.named_modules())
    placeholders: list[str] = []
    value: dict[fx.Node, str] = {}
    layers: list[LayerOp] = []
    graph_arg: fx.Node | None = None
    current: fx.Node | None = None

    def expect_current(node: fx.Node, arg) -> None:
        if arg is not current:
            raise NotImplementedError(
                f"{node.format_node()}: only a linear chain of GCNConv/GATConv/SAGEConv layers is supported"
            )

    def act_of(node: fx.Node) -> int | None:
        if node.op == "call_function" and node.target in _RELU:
            return rt.ACT_RELU
        if node.op == "call_method" and node.target == "relu":
            return rt.ACT_RELU
        if node.op == "call_module" and isinstance(modules[node.target], torch.nn.ReLU):
            return rt.ACT_RELU
        if node.op == "call_function" and node.target in _ELU:
            alpha = node.kwargs.get("alpha", node.args[1] if len(node.args) > 1 else 1.0)
            if alpha != 1.0:
                raise NotImplementedError("elu with alpha != 1")
            return rt.ACT_ELU
        if node.op == "call_module" and isinstance(modules[node.target], torch.nn.ELU):
            if modules[node.target].alpha != 1.0:
                raise NotImplementedError("elu with alpha != 1")
            return rt.ACT_ELU
        return None

    for node in gm.graph.nodes:
        if node.op == "placeholder":
            placeholders.append(node.target)
            if len(placeholders) == 1:
                current = node
            elif len(placeholders) == 2:
                graph_arg = node
            else:
                raise NotImplementedError("models take (x, adjacency or edge_index)")
            continue
        if node.op == "call_module" and _is_conv(modules[node.target]):
            expect_current(node, node.args[0])
            if len(node.args) < 2 or node.args[1] is not graph_arg or len(node.args) > 2 or node.kwargs:
                raise NotImplementedError(f"{node.target}: call it as conv(x, graph)")
            layers.append(_layer_from_module(node.target, modules[node.target]))
            current = node
            continue
        act = act_of(node)
        if act is not None:
            expect_current(node, node.args[0])
            if not layers or layers[-1].act != rt.ACT_NONE or layers[-1].log_softmax:
                raise NotImplementedError(f"{node.format_node()}: activation must follow a conv")
            layers[-1].act = act
            current = node
            continue
        if (node.op == "call_function" and node.target in _DROPOUT) or (
            node.op == "call_module" and isinstance(modules[node.target], torch.nn.Dropout)
        ):
            expect_current(node, node.args[0])
            training = node.kwargs.get("training", node.args[2] if len(node.args) > 2 else True)
            if node.op == "call_module":
                training = modules[node.target].training
            if training:
                raise NotImplementedError("dropout in training mode")
            current = node
            continue
        is_lsm = (node.op == "call_function" and node.target in _LOGSM) or (
            node.op == "call_method" and node.target == "log_softmax"
        )
        if is_lsm:
            expect_current(node, node.args[0])
            dim = node.kwargs.get("dim", node.args[1] if len(node.args) > 1 else None)
            if dim not in (-1, 1) or not layers:
                raise NotImplementedError("log_softmax must be over the feature dim after a conv")
            layers[-1].log_softmax = True
            current = node
            continue
        if node.op == "output":
            out = node.args[0]
            if isinstance(out, (tuple, list)):
                if len(out) != 1:
                    raise NotImplementedError("multi-output models are not supported")
                out = out[0]
            expect_current(node, out)
            continue
        if node.op == "call_function" and node.target is operator.getitem:
            raise NotImplementedError(f"{node.format_node()}: unsupported indexing")
        raise NotImplementedError(f"op {node.format_node()} is not supported by the b200 target")

    if not layers:
        raise NotImplementedError("no GCNConv/GATConv/SAGEConv layer found")
    for prev, nxt in zip(layers, layers[1:], strict=False):
        if prev.out_width != nxt.in_channels:
            raise ValueError(f"{nxt.name} expects {nxt.in_channels} features, gets {prev.out_width}")
    return B200Program(layers=layers, input_names=placeholders,
                       feature_dtype=feature_dtype or torch.float32,
                       output_dtype=output_dtype or torch.float32)


# ---------------------------------------------------------------------------
# Execution
# ---------------------------------------------------------------------------


@dataclass
class DeviceGraph:
    """A graph resident on one device in the layout the kernels read."""

    rowptr: torch.Tensor  # int32 [N+1]
    col: torch.Tensor  # int32 [E]
    w: torch.Tensor | None  # fp32 [E] (GCN weights) or None (GAT)
    plan: rt.Plan
    num_nodes: int
    cta_threshold: int = 0  # the plan's thresholds as given (0: the library's default)
    split_threshold: int = 0
    _chunks: dict = field(default_factory=dict, repr=False)

    @property
    def num_edges(self) -> int:
        return self.col.numel()

    def row_chunks(self, k: int) -> list[tuple[int, int, rt.Plan]]:
        """The rows split into k ranges of about equal edge counts, each with its
        own plan over the (un-rebased) rowptr slice; built once per k.

        Each chunk plan splits exactly the rows the whole graph's plan splits
        (the whole graph's split threshold, not the default a chunk's smaller
        edge count would give), so every row takes the same kernel path and
        the chunked result equals the single launch bit for bit."""
        got = self._chunks.get(k)
        if got is None:
            from gnnc.b200.partition import whole_graph_split_threshold

            n = self.rowptr.numel() - 1
            split = self.split_threshold or whole_graph_split_threshold(
                self.num_edges, torch.cuda.get_device_properties(self.rowptr.device)
                .multi_processor_count)
            targets = torch.linspace(0, self.num_edges, k + 1, device=self.rowptr.device)[1:-1]
            cuts = torch.searchsorted(self.rowptr, targets.to(torch.int32)).tolist()
            bounds = sorted({0, n, *(min(max(int(c), 0), n) for c in cuts)})
            got = [(a, b, rt.Plan(self.rowptr[a : b + 1], cta_threshold=self.cta_threshold,
                                  split_threshold=split))
                   for a, b in zip(bounds, bounds[1:]) if b > a]
            self._chunks[k] = got
        return got


def graph_from_csr(adj: torch.Tensor, device, *, cta_threshold=0, split_threshold=0) -> DeviceGraph:
    """Pre-normalised torch.sparse_csr adjacency -> DeviceGraph (values kept as weights).

    Follows the (crow_indices, col_indices, values) decomposition of
    gnnc/execution/__init__.py:72-100; indices are narrowed to int32."""
    crow = adj.crow_indices()
    col = adj.col_indices()
    if adj.size(0) != adj.size(1):
        raise ValueError("adjacency must be square")
    if col.numel() >= 2**31:
        raise ValueError("more than 2^31 edges")
    rowptr = crow.to(device=device, dtype=torch.int32, non_blocking=True).contiguous()
    col = col.to(device=device, dtype=torch.int32, non_blocking=True).contiguous()
    w = adj.values().to(device=device, dtype=torch.float32, non_blocking=True).contiguous()
    rt.validate_csr(rowptr, col, adj.size(1))
    plan = rt.Plan(rowptr, cta_threshold=cta_threshold, split_threshold=split_threshold)
    return DeviceGraph(rowptr, col, w, plan, adj.size(0), cta_threshold, split_threshold)


def graph_from_edge_index(
    edge_index: torch.Tensor,
    num_nodes: int,
    device,
    *,
    self_loops: bool,
    dedupe: bool,
    normalize: bool,
    cta_threshold: int = 0,
    split_threshold: int = 0,
) -> DeviceGraph:
    """edge_index [2,E] -> CSR by destination on the device (+ GCN weights)."""
    ei = edge_index.to(device=device, dtype=torch.int64, non_blocking=True)
    rowptr, col, mult = rt.csr_from_coo(ei, num_nodes, self_loops=self_loops, dedupe=dedupe)
    w = None
    if normalize:
        _, _, w = rt.gcn_norm(rowptr, col, mult)
    elif dedupe:
        w = mult.to(torch.float32)
    plan = rt.Plan(rowptr, cta_threshold=cta_threshold, split_threshold=split_threshold)
    return DeviceGraph(rowptr, col, w, plan, num_nodes, cta_threshold, split_threshold)


def to_device_features(x: torch.Tensor, dtype: torch.dtype, device) -> torch.Tensor:
    """Copies x into a row-padded (16-byte aligned rows) device buffer of `dtype`."""
    out = rt.empty_rows(x.size(0), x.size(1), dtype, device)
    out.copy_(x, non_blocking=True)
    return out


class _PinnedResults:
    """Page-locked host buffers for results, recycled across calls.

    Allocating page-locked memory costs about as much as the transfer it
    speeds up (hundreds of ms per GB), so results for host inputs are written
    into buffers kept here. A buffer is handed out again only when nothing but
    this pool references it (views and numpy arrays of a result keep it
    referenced), so a result the caller still holds is never overwritten.
    """

    def __init__(self, max_buffers: int = 4) -> None:
        self.max_buffers = max_buffers
        self.pool: dict[tuple, list[torch.Tensor]] = {}

    def take(self, shape: tuple, dtype: torch.dtype) -> torch.Tensor:
        bufs = self.pool.setdefault((tuple(shape), dtype), [])
        for buf in bufs:
            # references: the pool list, this loop variable, getrefcount's argument
            if sys.getrefcount(buf) <= 3:
                return buf
        buf = torch.empty(tuple(shape), dtype=dtype, pin_memory=True)
        if len(bufs) < self.max_buffers:
            bufs.append(buf)
        return buf


class B200Executable:
    """A lowered model bound to one CUDA device. Call with the forward inputs."""

    def __init__(self, program: B200Program, device: torch.device | str | None = None) -> None:
        self.program = program
        self.device = torch.device(device) if device is not None else torch.device(
            "cuda", torch.cuda.current_device()
        )
        dt = program.feature_dtype
        self._weights = []
        self._roots: list[torch.Tensor | None] = []
        for layer in program.layers:
            w = layer.weight.to(device=self.device, dtype=dt)
            w = to_device_features(w, dt, self.device)
            asrc = adst = None
            if layer.att_src is not None:
                asrc = layer.att_src.to(self.device, torch.float32).contiguous()
                adst = layer.att_dst.to(self.device, torch.float32).contiguous()
            bias = None if layer.bias is None else layer.bias.to(self.device, torch.float32)
            self._weights.append((w, asrc, adst, bias))
            wr = None
            if layer.weight_root is not None:
                wr = to_device_features(layer.weight_root.to(device=self.device, dtype=dt), dt,
                                        self.device)
            self._roots.append(wr)
        self._graphs: dict[tuple, tuple[object, DeviceGraph]] = {}
        self._results = _PinnedResults()
        self._copy_stream: torch.cuda.Stream | None = None
        self._in_stream: torch.cuda.Stream | None = None  # run_stream's input copies
        self._cuda_graphs: dict[tuple, tuple] = {}
        self.cuda_graph_error: str | None = None

    def __str__(self) -> str:
        return f"b200.executable(device={self.device})\n{self.program}"

    # Graphs are cached per (storage, shape, strides, version counter, layer
    # graph mode). detach() and views share the storage and the version counter,
    # so the same user tensor hits the cache on every call, while an in-place
    # update (version bump) rebuilds it. The cache holds the tensor, keeping its
    # storage (and address) alive.
    @staticmethod
    def _graph_key(graph: torch.Tensor) -> tuple:
        if graph.layout == torch.sparse_csr:
            parts = (graph.crow_indices(), graph.col_indices(), graph.values())
            return tuple((t.device, t.data_ptr(), tuple(t.shape), t._version) for t in parts)
        return (graph.device, graph.data_ptr(), tuple(graph.shape), tuple(graph.stride()),
                graph.dtype, graph._version)

    def _graph_for(self, graph: torch.Tensor, num_nodes: int, layer: LayerOp) -> DeviceGraph:
        if graph.layout == torch.sparse_csr:
            if layer.kind == "sage":
                mode = ("csr-mean",)
            elif layer.kind != "gcn" or layer.normalize:
                raise NotImplementedError(
                    "a sparse CSR adjacency must be pre-normalised for GCNConv(normalize=False)"
                )
            else:
                mode = ("csr",)
        elif graph.layout == torch.strided:
            if layer.kind == "gcn":
                mode = ("coo", layer.add_self_loops, True, layer.normalize)
            elif layer.kind == "sage":
                mode = ("coo-mean",)
            else:
                mode = ("coo", layer.add_self_loops, False, False)
        else:
            raise NotImplementedError(f"unsupported graph layout {graph.layout}")
        key = (self._graph_key(graph), num_nodes, *mode)
        hit = self._graphs.get(key)
        if hit is not None:
            return hit[1]
        if mode[0] == "csr":
            g = graph_from_csr(graph, self.device)
        elif mode[0] == "csr-mean":
            g = graph_from_csr(graph, self.device)
            g.w = rt.mean_norm(g.rowptr, g.w)
        elif mode[0] == "coo-mean":
            # SAGEConv on an edge list: no self-loops added, duplicates counted
            g = graph_from_edge_index(graph, num_nodes, self.device, self_loops=False,
                                      dedupe=False, normalize=False)
            g.w = rt.mean_norm(g.rowptr)
        else:
            g = graph_from_edge_index(
                graph, num_nodes, self.device, self_loops=mode[1], dedupe=mode[2], normalize=mode[3]
            )
        if len(self._graphs) > 4:
            self._graphs.clear()
        self._graphs[key] = (graph, g)
        return g

    # Results for host inputs leave the device while the last aggregation still
    # runs: its rows are aggregated in this many edge-balanced ranges, and each
    # range's rows are copied to the host on a side stream as soon as they are
    # done (graphs of at least this many edges per range; smaller ones use one).
    host_chunks = 8
    host_chunk_min_edges = 1 << 21

    def run_device(self, x: torch.Tensor, graph: torch.Tensor, events: list | None = None,
                   host_out=None, layer_outputs: list | None = None, staged: bool = False,
                   host_done: list | None = None) -> torch.Tensor:
        """Forward on device-resident (or host) inputs; returns the device output.

        events: if a list, receives per layer a (projection_start, aggregation_start,
        end) triple of recorded CUDA events (for per-layer timing).
        layer_outputs: if a list, receives each layer's device output rows in
        order (the last one is the result).
        host_out: if given, a callable (shape, dtype) -> page-locked host tensor;
        the result is copied into it (overlapped with the last aggregation) and
        the host tensor is returned once the copies are queued (synchronize the
        current stream before reading it).
        staged: x is already a device buffer of the feature dtype with 16-byte
        aligned rows (run_stream's input slots); it is read in place.
        host_done: with host_out, if a list, receives an event recorded after the
        result's copies instead of the current stream waiting for them."""
        dt = self.program.feature_dtype
        n = x.size(0)
        h_in = x if staged else to_device_features(x, dt, self.device)
        layers = self.program.layers
        with torch.cuda.device(self.device):
            for i, (layer, (w, asrc_w, adst_w, bias), wr) in enumerate(
                zip(layers, self._weights, self._roots, strict=True)
            ):
                g = self._graph_for(graph, n, layer)
                ev = None
                if events is not None:
                    ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
                    ev[0].record()
                    events.append(ev)
                last = i == len(layers) - 1
                out_dtype = self.program.output_dtype if last else dt
                root = None
                if layer.kind == "gcn":
                    h = rt.proj(h_in, w, out_dtype=dt)
                    asrc = adst = None
                    width = h.size(1)
                elif layer.kind == "sage":
                    h = rt.proj(h_in, w, out_dtype=dt)
                    root = rt.proj(h_in, wr, out_dtype=dt)
                    asrc = adst = None
                    width = h.size(1)
                else:
                    h, asrc, adst = rt.proj(h_in, w, att_src=asrc_w, att_dst=adst_w,
                                            heads=layer.heads, out_dtype=dt)
                    width = h.size(1) if layer.concat else h.size(1) // layer.heads
                if ev:
                    ev[1].record()
                out = rt.empty_rows(n, width, out_dtype, self.device)
                if last and host_out is not None:
                    host = host_out((n, width), out_dtype)
                    self._aggregate_to_host(layer, g, h, asrc, adst, bias, out, host, root,
                                            host_done)
                    h_in = host
                else:
                    self._aggregate(layer, g, g.plan, 0, n, h, asrc, adst, bias, out, root)
                    h_in = out
                if layer_outputs is not None:
                    layer_outputs.append(out)
                if ev:
                    ev[2].record()
        return h_in

    @staticmethod
    def _aggregate(layer, g, plan, r0, r1, h, asrc, adst, bias, out, root=None) -> None:
        """Aggregate destination rows [r0, r1) (plan covers exactly those rows)."""
        rowptr = g.rowptr[r0 : r1 + 1]
        if layer.kind == "sage":
            rt.sage_aggregate(plan, rowptr, g.col, g.w, h, root[r0:r1], bias=bias, act=layer.act,
                              log_softmax=layer.log_softmax, out_dtype=out.dtype, out=out[r0:r1])
        elif layer.kind == "gcn":
            rt.gcn_aggregate(plan, rowptr, g.col, g.w, h, bias=bias, act=layer.act,
                             log_softmax=layer.log_softmax, out_dtype=out.dtype,
                             out=out[r0:r1], n_src=h.size(0))
        else:
            rt.gat_aggregate(plan, rowptr, g.col, h, asrc, adst[r0:r1], heads=layer.heads,
                             negative_slope=layer.negative_slope, concat=layer.concat,
                             bias=bias, act=layer.act, log_softmax=layer.log_softmax,
                             out_dtype=out.dtype, out=out[r0:r1])

    def _aggregate_to_host(self, layer, g, h, asrc, adst, bias, out, host, root=None,
                           host_done: list | None = None) -> None:
        k = self.host_chunks if g.num_edges >= self.host_chunks * self.host_chunk_min_edges else 1
        cur = torch.cuda.current_stream(self.device)
        if self._copy_stream is None:
            self._copy_stream = torch.cuda.Stream(self.device)
        side = self._copy_stream
        chunks = g.row_chunks(k) if k > 1 else [(0, g.num_nodes, g.plan)]
        for r0, r1, plan in chunks:
            self._aggregate(layer, g, plan, r0, r1, h, asrc, adst, bias, out, root)
            done = torch.cuda.Event()
            done.record(cur)
            side.wait_event(done)
            with torch.cuda.stream(side):
                host[r0:r1].copy_(out[r0:r1], non_blocking=True)
        out.record_stream(side)
        if host_done is None:
            cur.wait_stream(side)
        else:
            done = torch.cuda.Event()
            done.record(side)
            host_done.append(done)

    def run_stream(self, batches, graph: torch.Tensor):
        """Forwards of a stream of batches of host input rows, pipelined.

        For callers that feed many batches through one GPU over PCIe, where a
        call at a time leaves one copy direction idle: batch k+1's input rows
        go to the device on one copy engine while batch k computes and its
        result rows come back on the other (the result copies overlap the last
        aggregation as in __call__). `batches` yields host tensors [N, in]
        (page-locked ones copy at full rate). Yields each batch's result, a
        page-locked host tensor as __call__ returns for host inputs, once its
        copies completed; a result the caller keeps is never overwritten.
        Runs eagerly (no CUDA-graph replay) and equals __call__ row for row."""
        it = iter(batches)
        x = next(it, None)
        if x is None:
            return
        dev, dt = self.device, self.program.feature_dtype
        cur = torch.cuda.current_stream(dev)
        if self._in_stream is None:
            self._in_stream = torch.cuda.Stream(dev)
        ins = self._in_stream
        slots: list[torch.Tensor | None] = [None, None]
        freed: list[torch.cuda.Event | None] = [None, None]  # the slot's last forward done

        def stage(x: torch.Tensor, b: int):
            if x.is_cuda:
                raise ValueError("run_stream takes host batches")
            n, c = x.shape
            buf = slots[b]
            if buf is None or tuple(buf.shape) != (n, c):
                buf = slots[b] = rt.empty_rows(n, c, dt, dev)
                buf.record_stream(ins)
            if freed[b] is not None:
                ins.wait_event(freed[b])
            with torch.cuda.stream(ins):
                buf.copy_(x, non_blocking=True)
                ready = torch.cuda.Event()
                ready.record(ins)
            return buf, ready

        with torch.cuda.device(dev):
            staged = stage(x, 0)
            pending = None
            k = 0
            while staged is not None:
                buf, ready = staged
                nxt = next(it, None)
                cur.wait_event(ready)
                done: list = []
                host = self.run_device(buf, graph, host_out=self._results.take, staged=True,
                                       host_done=done)
                ev = torch.cuda.Event()
                ev.record(cur)
                freed[k % 2] = ev
                staged = stage(nxt, (k + 1) % 2) if nxt is not None else None
                if pending is not None:
                    pending[1].synchronize()
                    yield pending[0]
                pending = (host, done[0])
                k += 1
            pending[1].synchronize()
            yield pending[0]

    def graph_edges(self, graph: torch.Tensor, num_nodes: int) -> list[int]:
        """Stored edges (self-loops included) each layer aggregates over."""
        return [self._graph_for(graph, num_nodes, layer).num_edges for layer in self.program.layers]

    # Small graphs are launch-bound: their forward is captured once into a
    # CUDA graph (per graph tensor and input shape) and replayed, so a call
    # costs one graph launch instead of a dozen kernel launches and their
    # Python wrappers. Graphs with at least this many stored edges run eagerly.
    cuda_graph_max_edges = 1 << 22

    def _replay(self, x: torch.Tensor, graph: torch.Tensor) -> torch.Tensor | None:
        """Forward through a captured CUDA graph; None when not applicable."""
        if self.cuda_graph_error is not None:
            return None
        n = x.size(0)
        if sum(self._graph_for(graph, n, layer).num_edges for layer in self.program.layers) >= (
            self.cuda_graph_max_edges * len(self.program.layers)
        ):
            return None
        key = (self._graph_key(graph), tuple(x.shape), x.dtype)
        entry = self._cuda_graphs.get(key)
        if entry is None:
            try:
                static_x = torch.empty(tuple(x.shape), dtype=x.dtype, device=self.device)
                static_x.copy_(x)
                self.run_device(static_x, graph)  # plans, workspace, module loading
                torch.cuda.synchronize(self.device)
                cg = torch.cuda.CUDAGraph()
                with torch.cuda.graph(cg):
                    static_out = self.run_device(static_x, graph)
                entry = (cg, static_x, static_out)
            except RuntimeError as exc:  # capture refused: run eagerly from now on
                self.cuda_graph_error = str(exc)
                return None
            if len(self._cuda_graphs) > 4:
                self._cuda_graphs.clear()
            self._cuda_graphs[key] = entry
        cg, static_x, static_out = entry
        static_x.copy_(x, non_blocking=True)
        cg.replay()
        return static_out

    def __call__(self, *inputs: torch.Tensor) -> list[torch.Tensor]:
        if len(inputs) != 2:
            raise ValueError(f"expected (x, graph) inputs, got {len(inputs)}")
        x, graph = inputs
        out = self._replay(x, graph)
        if out is not None:
            if not x.is_cuda:
                host = self._results.take(tuple(out.shape), out.dtype)
                host.copy_(out, non_blocking=True)
                torch.cuda.current_stream(self.device).synchronize()
                return [host]
            return [out.clone()]
        if not x.is_cuda:
            # Page-locked result buffer: the copies run as DMAs at full rate,
            # overlapped with the last aggregation.
            host = self.run_device(x, graph, host_out=self._results.take)
            torch.cuda.current_stream(self.device).synchronize()
            return [host]
        out = self.run_device(x, graph)
        return [out.contiguous()]
