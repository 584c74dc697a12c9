"""PyG-compatible GCNConv / GATConv / SAGEConv layers for environments without torch_geometric.

The reference's models are stock PyG layers (gnnc/examples/models/gcn.py:23,36-37;
experiments/pyg-baseline/run.py:47,78-88). These classes keep PyG's parameter
names, shapes and initialisation order, so a model built here under
`torch.manual_seed(s)` holds exactly the weights PyG would give it: the `lin`
weight is glorot-initialised twice (once by Linear's constructor, once by the
conv's reset_parameters), then att_src, att_dst, then zero bias. The weights
embedded in test/reference/gcn.raw.mlir and
experiments/gatconv/dumps/gat.1-raw-torch.mlir:137-139 reproduce bit for bit.
SAGEConv's lin_l / lin_r use PyG Linear's default initialisation (kaiming
uniform with a = sqrt(5), bias uniform in +-1/sqrt(fan_in)), drawn once by each
Linear's constructor and again by the conv's reset_parameters; the weights in
test/reference/sage.raw.mlir reproduce bit for bit.

`forward` is the eager PyTorch definition of the layer (the semantics
`gnnc-bench` compares against). The B200 path never calls it:
`gnnc.compile.compile_executable(..., target="b200")` reads the parameters and
runs the CUDA kernels instead.
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F
from torch import Tensor, nn

__all__ = ["GATConv", "GCNConv", "Linear", "SAGEConv", "glorot", "gcn_norm_edges", "spmm_mean"]


def glorot(t: Tensor | None) -> None:
    """U(-a, a), a = sqrt(6 / (fan_in + fan_out)) over the last two dims (PyG inits.glorot)."""
    if t is None:
        return
    a = math.sqrt(6.0 / (t.size(-2) + t.size(-1)))
    with torch.no_grad():
        t.uniform_(-a, a)


def _zeros(t: Tensor | None) -> None:
    if t is not None:
        with torch.no_grad():
            t.zero_()


class Linear(nn.Module):
    """torch_geometric.nn.dense.Linear: weight_initializer='glorot' (zero bias,
    as GCNConv / GATConv build it) or None (PyG's default: kaiming uniform,
    bias uniform in +-1/sqrt(in_channels), as SAGEConv builds it)."""

    def __init__(self, in_channels: int, out_channels: int, bias: bool = True,
                 weight_initializer: str | None = "glorot") -> None:
        super().__init__()
        self.in_channels = in_channels
        self.out_channels = out_channels
        self.weight_initializer = weight_initializer
        self.weight = nn.Parameter(torch.empty(out_channels, in_channels))
        if bias:
            self.bias = nn.Parameter(torch.empty(out_channels))
        else:
            self.register_parameter("bias", None)
        self.reset_parameters()

    def reset_parameters(self) -> None:
        if self.weight_initializer == "glorot":
            glorot(self.weight)
            _zeros(self.bias)
            return
        # PyG inits.kaiming_uniform(fan=in_channels, a=sqrt(5)) and inits.uniform
        bound = math.sqrt(6.0 / ((1.0 + 5.0) * self.in_channels))
        with torch.no_grad():
            self.weight.uniform_(-bound, bound)
            if self.bias is not None:
                b = 1.0 / math.sqrt(self.in_channels)
                self.bias.uniform_(-b, b)

    def forward(self, x: Tensor) -> Tensor:
        return F.linear(x, self.weight, self.bias)


def gcn_norm_edges(
    edge_index: Tensor, num_nodes: int, add_self_loops: bool = True, dtype=torch.float32
) -> tuple[Tensor, Tensor]:
    """PyG gcn_norm on an edge list with unit weights (flow source_to_target).

    add_remaining_self_loops drops every existing (i, i) edge and appends one
    loop per node; deg counts incoming edges (duplicates included); the edge
    weight is dinv[src] * 1 * dinv[dst] with dinv = deg^-1/2 (inf -> 0).
    """
    if add_self_loops:
        keep = edge_index[0] != edge_index[1]
        loops = torch.arange(num_nodes, device=edge_index.device, dtype=edge_index.dtype)
        edge_index = torch.cat([edge_index[:, keep], torch.stack([loops, loops])], dim=1)
    w = torch.ones(edge_index.size(1), dtype=dtype, device=edge_index.device)
    src, dst = edge_index[0], edge_index[1]
    deg = torch.zeros(num_nodes, dtype=dtype, device=edge_index.device).scatter_add_(0, dst, w)
    dinv = deg.pow_(-0.5)
    dinv.masked_fill_(dinv == float("inf"), 0)
    return edge_index, dinv[src] * w * dinv[dst]


class GCNConv(nn.Module):
    """PyG GCNConv: out = A_hat . (x W^T) + b."""

    def __init__(
        self,
        in_channels: int,
        out_channels: int,
        improved: bool = False,
        cached: bool = False,
        add_self_loops: bool | None = None,
        normalize: bool = True,
        bias: bool = True,
    ) -> None:
        super().__init__()
        if add_self_loops is None:
            add_self_loops = normalize
        self.in_channels = in_channels
        self.out_channels = out_channels
        self.improved = improved
        self.cached = cached
        self.add_self_loops = add_self_loops
        self.normalize = normalize
        self.lin = Linear(in_channels, out_channels, bias=False)
        if bias:
            self.bias = nn.Parameter(torch.empty(out_channels))
        else:
            self.register_parameter("bias", None)
        self.reset_parameters()

    def reset_parameters(self) -> None:
        self.lin.reset_parameters()
        _zeros(self.bias)

    def forward(self, x: Tensor, edge_index: Tensor, edge_weight: Tensor | None = None) -> Tensor:
        if self.improved:
            raise NotImplementedError("improved=True is not supported")
        x = self.lin(x)
        if edge_index.layout == torch.sparse_csr:
            if self.normalize:
                raise NotImplementedError("pass a pre-normalised CSR with normalize=False")
            out = torch.sparse.mm(edge_index, x)
        else:
            n = x.size(0)
            if self.normalize:
                edge_index, w = gcn_norm_edges(edge_index, n, self.add_self_loops, x.dtype)
            else:
                w = torch.ones(edge_index.size(1), dtype=x.dtype, device=x.device)
                if edge_weight is not None:
                    w = edge_weight
            out = torch.zeros_like(x).index_add_(0, edge_index[1], x[edge_index[0]] * w[:, None])
        if self.bias is not None:
            out = out + self.bias
        return out


class GATConv(nn.Module):
    """PyG GATConv (single edge type, no edge features, no residual)."""

    def __init__(
        self,
        in_channels: int,
        out_channels: int,
        heads: int = 1,
        concat: bool = True,
        negative_slope: float = 0.2,
        dropout: float = 0.0,
        add_self_loops: bool = True,
        edge_dim: int | None = None,
        fill_value: str = "mean",
        bias: bool = True,
        residual: bool = False,
    ) -> None:
        super().__init__()
        if edge_dim is not None or residual:
            raise NotImplementedError("edge features and residual connections are not supported")
        self.in_channels = in_channels
        self.out_channels = out_channels
        self.heads = heads
        self.concat = concat
        self.negative_slope = negative_slope
        self.dropout = dropout
        self.add_self_loops = add_self_loops
        self.edge_dim = None
        self.residual = False
        self.lin = Linear(in_channels, heads * out_channels, bias=False)
        self.att_src = nn.Parameter(torch.empty(1, heads, out_channels))
        self.att_dst = nn.Parameter(torch.empty(1, heads, out_channels))
        if bias and concat:
            self.bias = nn.Parameter(torch.empty(heads * out_channels))
        elif bias:
            self.bias = nn.Parameter(torch.empty(out_channels))
        else:
            self.register_parameter("bias", None)
        self.reset_parameters()

    def reset_parameters(self) -> None:
        self.lin.reset_parameters()
        glorot(self.att_src)
        glorot(self.att_dst)
        _zeros(self.bias)

    def forward(self, x: Tensor, edge_index: Tensor) -> Tensor:
        H, C = self.heads, self.out_channels
        n = x.size(0)
        h = self.lin(x).view(-1, H, C)
        a_src = (h * self.att_src).sum(dim=-1)
        a_dst = (h * self.att_dst).sum(dim=-1)
        if self.add_self_loops:
            keep = edge_index[0] != edge_index[1]
            loops = torch.arange(n, device=x.device, dtype=edge_index.dtype)
            edge_index = torch.cat([edge_index[:, keep], torch.stack([loops, loops])], dim=1)
        src, dst = edge_index[0], edge_index[1]
        e = F.leaky_relu(a_src.index_select(0, src) + a_dst.index_select(0, dst), self.negative_slope)
        idx = dst.view(-1, 1).expand_as(e)
        m = e.new_zeros((n, H)).scatter_reduce(0, idx, e.detach(), "amax", include_self=False)
        p = (e - m.index_select(0, dst)).exp()
        s = e.new_zeros((n, H)).scatter_add(0, idx, p) + 1e-16
        alpha = p / s.index_select(0, dst)
        alpha = F.dropout(alpha, p=self.dropout, training=self.training)
        msg = h.index_select(0, src) * alpha.unsqueeze(-1)
        out = h.new_zeros((n, H, C)).index_add_(0, dst, msg)
        out = out.view(-1, H * C) if self.concat else out.mean(dim=1)
        if self.bias is not None:
            out = out + self.bias
        return out


def spmm_mean(adj: Tensor, x: Tensor) -> Tensor:
    """(A . x) / clamp_min(row_nnz, 1) over a sparse CSR adjacency, row_nnz the
    number of nonzero stored values of the row (the reference's
    `_sparse_mm.reduce("mean")` rewrite,
    gnnc/conversion/tm_tensor_to_torch/despecialize_sparse_mm_reduce.py:1-75)."""
    crow = adj.crow_indices()
    vals = adj.values()
    rows = torch.repeat_interleave(torch.arange(crow.numel() - 1, device=x.device), crow.diff())
    nnz = torch.zeros(crow.numel() - 1, dtype=x.dtype, device=x.device).index_add_(
        0, rows, (vals != 0).to(x.dtype))
    return (adj.to(x.dtype) @ x) / nnz.clamp_min(1.0).unsqueeze(1)


class SAGEConv(nn.Module):
    """PyG SAGEConv(in, out) with the defaults (aggr='mean', root_weight=True,
    normalize=False, project=False, bias=True):

        out = lin_l(mean_{j in N(i)} x_j) + lin_r(x_i)

    On a torch.sparse_csr adjacency the mean is spmm_mean (values used, rows
    divided by their count of nonzero values), as the reference's SAGE model
    feeds it (gnnc/examples/models/sage.py; test/reference/sage.raw.mlir:5-14).
    On an edge_index [2, E] the mean is over incoming edges (duplicates counted)."""

    def __init__(self, in_channels: int, out_channels: int, bias: bool = True) -> None:
        super().__init__()
        self.in_channels = in_channels
        self.out_channels = out_channels
        self.aggr = "mean"
        self.root_weight = True
        self.normalize = False
        self.lin_l = Linear(in_channels, out_channels, bias=bias, weight_initializer=None)
        self.lin_r = Linear(in_channels, out_channels, bias=False, weight_initializer=None)
        self.reset_parameters()

    def reset_parameters(self) -> None:
        self.lin_l.reset_parameters()
        self.lin_r.reset_parameters()

    def forward(self, x: Tensor, graph: Tensor) -> Tensor:
        if graph.layout == torch.sparse_csr:
            aggr = spmm_mean(graph, x)
        else:
            src, dst = graph[0], graph[1]
            n = x.size(0)
            deg = torch.zeros(n, dtype=x.dtype, device=x.device).index_add_(
                0, dst, torch.ones_like(dst, dtype=x.dtype))
            aggr = torch.zeros_like(x).index_add_(0, dst, x.index_select(0, src))
            aggr = aggr / deg.clamp_min(1.0).unsqueeze(1)
        return self.lin_l(aggr) + self.lin_r(x)
