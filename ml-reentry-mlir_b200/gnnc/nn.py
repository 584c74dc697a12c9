"""PyG-compatible GCNConv / GATConv layers for environments without torch_geometric.

The reference's models are stock PyG layers (gnnc/examples/models/gcn.py:23,36-37;
experiments/pyg-baseline/run.py:47,78-88). These classes keep PyG's parameter
names, shapes and initialisation order, so a model built here under
`torch.manual_seed(s)` holds exactly the weights PyG would give it: the `lin`
weight is glorot-initialised twice (once by Linear's constructor, once by the
conv's reset_parameters), then att_src, att_dst, then zero bias. The weights
embedded in test/reference/gcn.raw.mlir and
experiments/gatconv/dumps/gat.1-raw-torch.mlir:137-139 reproduce bit for bit.

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

__all__ = ["GATConv", "GCNConv", "Linear", "glorot", "gcn_norm_edges"]


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
    """torch_geometric.nn.dense.Linear with weight_initializer='glorot'."""

    def __init__(self, in_channels: int, out_channels: int, bias: bool = True) -> None:
        super().__init__()
        self.in_channels = in_channels
        self.out_channels = out_channels
        self.weight = nn.Parameter(torch.empty(out_channels, in_channels))
        if bias:
            self.bias = nn.Parameter(torch.empty(out_channels))
        else:
            self.register_parameter("bias", None)
        self.reset_parameters()

    def reset_parameters(self) -> None:
        glorot(self.weight)
        _zeros(self.bias)

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
