"""CPU oracle for the GCN / GAT aggregation path (TEST INFRASTRUCTURE ONLY).

This module is the checker, never the product: only tests/, the smoke check in
__graft_entry__.py and bench.py's CPU-baseline leg may import it. The B200
path (gnnc.compile / gnnc.execution / libgnnc_b200.so) never calls it.

What it restates. The reference's hot path is GCNConv's CSR SpMM and GATConv's
SDDMM -> LeakyReLU -> edge softmax -> SpMM chain. Its arithmetic lives in the
third-party PyTorch Geometric package (torch-geometric >= 2.5, measured on
2.7.0 per experiments/pyg-baseline/README.md:19-27; torch_scatter pinned at
edeb0422, torch_sparse at 2be752eb, third_party/README.md:13-14), none of
which is installed here, so this file restates the published algorithms in
plain PyTorch CPU ops, following the reference's own call sites:

  gcn_norm              <- gnnc/examples/util.py:16-41 (call site :22) and PyG gcn_norm
  normalized_csr_adj    <- gnnc/examples/util.py:16-41 (flip, coalesce, to_sparse_csr)
  csr_from_coo          <- the same ordering, restated in numpy (integer work)
  spmm_csr / gcn_layer  <- test/reference/gcn.raw.mlir:4-21, gcn.linalg-on-tensors.mlir:19-26
  gat_layer             <- experiments/gatconv/dumps/gat.1-raw-torch.mlir:5-129, op by op
  softmax_aggregate     <- experiments/gat-gpu-codegen/gat-kernel.mlir:31-132
  gat_rows_fp64         <- the same GAT math, chunked over destination rows in
                           float64 for graphs whose E x H x C messages do not fit
  gat_layer_sample /    <- the same op sequence on a row range, the timed CPU
  gat_aggregate_sample     baseline (with / without the projection)
  spmm_mean / sage_layer <- test/reference/sage.raw.mlir:5-27 and the mean rewrite
                           gnnc/conversion/tm_tensor_to_torch/despecialize_sparse_mm_reduce.py:1-75

Pinning. tests/test_oracle_golden.py checks this oracle against every known
answer the reference carries for the path: the GCN and GATConv weight blobs
(test/reference/gcn.raw.mlir:26-35, experiments/gatconv/dumps/gat.1-raw-torch.mlir:137-139,
reproduced bit for bit by seeded initialisation), the softmax + SpMM output
(experiments/gat-gpu-codegen/dumps/cpu.out.txt) and the two SpMM outputs
(experiments/sparsifier-coo-check/dumps/01-spmm-csr.out.txt, 05-spmm-weighted-csr.out.txt).
No reference test pins PyG GCN/GAT output values on a real graph (its goldens
are computed live from eager PyG, test/integration/test_compile_matches_torch.py:50-53),
so whole-model outputs are pinned only through these fixtures and structure.
"""

from __future__ import annotations

import numpy as np
import torch
import torch.nn.functional as F

# ---------------------------------------------------------------------------
# Graph preparation (integer work is bit-exact)
# ---------------------------------------------------------------------------


def gcn_norm(edge_index: torch.Tensor, num_nodes: int, add_self_loops: bool = True):
    """PyG gcn_norm(edge_index, num_nodes, add_self_loops=True) with unit weights.

    add_remaining_self_loops: drop every (i,i) edge, append one loop per node.
    deg[dst] += 1 per edge (flow source_to_target); dinv = deg.pow(-0.5) with
    inf -> 0; w = dinv[src] * 1 * dinv[dst] in fp32 (util.py:22)."""
    if add_self_loops:
        keep = edge_index[0] != edge_index[1]
        loops = torch.arange(num_nodes, dtype=edge_index.dtype)
        edge_index = torch.cat([edge_index[:, keep], torch.stack([loops, loops])], dim=1)
    ones = torch.ones(edge_index.size(1), dtype=torch.float32)
    deg = torch.zeros(num_nodes, dtype=torch.float32).scatter_add_(0, edge_index[1], ones)
    dinv = deg.pow_(-0.5)
    dinv.masked_fill_(dinv == float("inf"), 0)
    return edge_index, dinv[edge_index[0]] * ones * dinv[edge_index[1]]


def normalized_csr_adj(edge_index: torch.Tensor, num_nodes: int):
    """util.py:16-41: sparse_coo_tensor(ei.flip(0), ew).coalesce().to_sparse_csr().

    Returns (crow int64 [N+1], col int64 [E], val fp32 [E])."""
    ei, ew = gcn_norm(edge_index, num_nodes)
    with torch.sparse.check_sparse_tensor_invariants(False):
        coo = torch.sparse_coo_tensor(ei.flip(0), ew, (num_nodes, num_nodes))
        csr = coo.coalesce().to_sparse_csr()
    return csr.crow_indices(), csr.col_indices(), csr.values()


def csr_from_coo(edge_index, num_nodes: int, *, self_loops: bool, dedupe: bool):
    """numpy restatement of the CSR build: rows = dst, cols = src ascending.

    self_loops drops every (i,i) edge and adds one per node; dedupe merges
    equal (dst,src) pairs (coalesce) and reports their multiplicity.
    Returns (rowptr int64 [N+1], col int64 [E'], mult int64 [E'])."""
    ei = np.asarray(edge_index, dtype=np.int64)
    src, dst = ei[0], ei[1]
    if self_loops:
        keep = src != dst
        loops = np.arange(num_nodes, dtype=np.int64)
        src = np.concatenate([src[keep], loops])
        dst = np.concatenate([dst[keep], loops])
    order = np.lexsort((src, dst))
    src, dst = src[order], dst[order]
    if dedupe and src.size:
        start = np.ones(src.size, dtype=bool)
        start[1:] = (src[1:] != src[:-1]) | (dst[1:] != dst[:-1])
        idx = np.flatnonzero(start)
        mult = np.diff(np.append(idx, src.size))
        src, dst = src[idx], dst[idx]
    else:
        mult = np.ones(src.size, dtype=np.int64)
    rowptr = np.zeros(num_nodes + 1, dtype=np.int64)
    np.add.at(rowptr, dst + 1, 1)
    return np.cumsum(rowptr), src, mult


def gcn_weights(rowptr, col, mult):
    """gcn_norm weights on a CSR that already has its loops (fp32, sequential sums)."""
    rowptr = np.asarray(rowptr)
    n = rowptr.size - 1
    deg = np.zeros(n, dtype=np.int64)
    rows = np.repeat(np.arange(n), np.diff(rowptr))
    np.add.at(deg, rows, np.asarray(mult))
    dinv = torch.from_numpy(deg.astype(np.float32)).pow_(-0.5)
    dinv.masked_fill_(dinv == float("inf"), 0)
    dinv = dinv.numpy()
    one = dinv[np.asarray(col)] * dinv[rows]
    w = one.copy()
    m = np.asarray(mult)
    for k in np.flatnonzero(m > 1):
        acc = np.float32(one[k])
        for _ in range(int(m[k]) - 1):
            acc = np.float32(acc + one[k])
        w[k] = acc
    return deg.astype(np.float32), dinv, w


# ---------------------------------------------------------------------------
# Layers
# ---------------------------------------------------------------------------


def _act(x: torch.Tensor, act: str | None) -> torch.Tensor:
    if act == "relu":
        return F.relu(x)
    if act == "elu":
        return F.elu(x)
    return x


def spmm_csr(crow, col, val, h: torch.Tensor) -> torch.Tensor:
    """out[i] = sum_k val[k] * h[col[k]] over row i, in CSR order (the sparsifier's loop)."""
    crow = torch.as_tensor(crow, dtype=torch.int64)
    col = torch.as_tensor(col, dtype=torch.int64)
    val = torch.as_tensor(val, dtype=h.dtype)
    rows = torch.repeat_interleave(torch.arange(crow.numel() - 1), crow.diff())
    out = torch.zeros((crow.numel() - 1, h.size(1)), dtype=h.dtype)
    return out.index_add_(0, rows, h.index_select(0, col) * val[:, None])


def gcn_layer(x, crow, col, val, weight, bias=None, act=None, log_softmax=False):
    """GCNConv(normalize=False): linear (no bias) -> _sparse_mm -> +bias (gcn.raw.mlir:6-10)."""
    h = x @ weight.t()
    out = spmm_csr(crow, col, val, h)
    if bias is not None:
        out = out + bias
    out = _act(out, act)
    return F.log_softmax(out, dim=-1) if log_softmax else out


def spmm_mean(crow, col, val, x):
    """_sparse_mm.reduce("mean"): (A . x) / clamp_min(row_nnz, 1), row_nnz = the row's
    count of nonzero values (despecialize_sparse_mm_reduce.py:1-75)."""
    crow = torch.as_tensor(crow, dtype=torch.int64)
    val = torch.as_tensor(val, dtype=x.dtype)
    rows = torch.repeat_interleave(torch.arange(crow.numel() - 1), crow.diff())
    nnz = x.new_zeros(crow.numel() - 1).index_add_(0, rows, (val != 0).to(x.dtype))
    return spmm_csr(crow, col, val, x) / nnz.clamp_min(1.0).unsqueeze(1)


def mean_weights(crow, val=None):
    """Edge weights val / max(row count of nonzero val, 1) in float32 with IEEE
    division: the exact values gnnc_mean_norm produces (val None: unit weights)."""
    crow = torch.as_tensor(crow, dtype=torch.int64)
    E = int(crow[-1])
    val = torch.ones(E, dtype=torch.float32) if val is None else torch.as_tensor(val, dtype=torch.float32)
    rows = torch.repeat_interleave(torch.arange(crow.numel() - 1), crow.diff())
    nnz = torch.zeros(crow.numel() - 1, dtype=torch.int64).index_add_(0, rows, (val != 0).long())
    return val / nnz.clamp_min(1).to(torch.float32)[rows]


def sage_layer(x, crow, col, val, weight_l, bias_l, weight_r, act=None, log_softmax=False):
    """PyG SAGEConv (mean, root weight) as the reference lowers it
    (sage.raw.mlir:5-14): mean-aggregate x, linear with bias, plus a linear of x
    without bias, then the activation."""
    out = spmm_mean(crow, col, val, x) @ weight_l.t()
    if bias_l is not None:
        out = out + bias_l
    out = out + x @ weight_r.t()
    out = _act(out, act)
    return F.log_softmax(out, dim=-1) if log_softmax else out


def gat_layer(
    x, edge_index, weight, att_src, att_dst, bias, heads: int, channels: int, *,
    concat=True, negative_slope=0.2, add_self_loops=True, act=None, log_softmax=False,
):
    """One PyG GATConv layer, op by op from gat.1-raw-torch.mlir."""
    H, C = heads, channels
    n = x.size(0)
    h = (x @ weight.t()).view(-1, H, C)  # :5-10 linear + view
    a_src = (h * att_src.view(1, H, C)).sum(dim=-1)  # :11-17
    a_dst = (h * att_dst.view(1, H, C)).sum(dim=-1)  # :18-24
    if add_self_loops:  # GATConv: remove_self_loops + add_self_loops
        keep = edge_index[0] != edge_index[1]
        loops = torch.arange(n, dtype=edge_index.dtype)
        edge_index = torch.cat([edge_index[:, keep], torch.stack([loops, loops])], dim=1)
    src, dst = edge_index[0], edge_index[1]  # :25-28 (select 0 -> src, 1 -> dst)
    e = a_src.index_select(0, src) + a_dst.index_select(0, dst)  # :29-36
    e = F.leaky_relu(e, negative_slope)  # :37-38
    idx = dst.view(-1, 1).expand_as(e)
    m = e.new_zeros((n, H)).scatter_reduce(0, idx, e.detach(), "amax", include_self=False)  # :39-60
    p = (e - m.index_select(0, dst)).exp()  # :61-65
    s = e.new_zeros((n, H)).scatter_add(0, idx, p) + 1e-16  # :66-87
    alpha = p / s.index_select(0, dst)  # :88-90
    msg = alpha.unsqueeze(-1) * h.index_select(0, src)  # :95-103
    out = h.new_zeros((n, H, C)).scatter_add(0, dst.view(-1, 1, 1).expand_as(msg), msg)  # :104-125
    out = out.view(-1, H * C) if concat else out.mean(dim=1)  # :126-129 / concat=False
    if bias is not None:
        out = out + bias
    out = _act(out, act)
    return F.log_softmax(out, dim=-1) if log_softmax else out


def softmax_aggregate(crow, col, scores, h, eps: float = 0.0):
    """out[i] = sum_k exp(s_k - max_i) / (sum exp(s - max_i) + eps) * h[col_k] (gat-kernel.mlir:31-132)."""
    crow = torch.as_tensor(crow, dtype=torch.int64)
    col = torch.as_tensor(col, dtype=torch.int64)
    s = torch.as_tensor(scores, dtype=h.dtype)
    n = crow.numel() - 1
    rows = torch.repeat_interleave(torch.arange(n), crow.diff())
    m = s.new_zeros(n).scatter_reduce(0, rows, s, "amax", include_self=False)
    p = (s - m[rows]).exp()
    den = s.new_zeros(n).scatter_add(0, rows, p) + eps
    a = p / den[rows]
    return h.new_zeros((n, h.size(1))).index_add_(0, rows, h.index_select(0, col) * a[:, None])


def gat_rows_fp64(
    rowptr, col, h, asrc, adst, heads: int, *, rows=None, negative_slope=0.2,
    concat=True, bias=None, act=None, log_softmax=False, chunk_edges=1 << 20,
):
    """The GAT aggregation of given h [N,H*C], asrc/adst [N,H] in float64, for the
    destination rows `rows` (default all), chunked so memory stays bounded.
    Returns [len(rows), F_out] float64."""
    rowptr = torch.as_tensor(rowptr, dtype=torch.int64)
    col = torch.as_tensor(col, dtype=torch.int64)
    n = rowptr.numel() - 1
    rows = torch.arange(n) if rows is None else torch.as_tensor(rows, dtype=torch.int64)
    H = heads
    Fw = h.size(1)
    C = Fw // H
    outs = []
    i = 0
    while i < rows.numel():
        # grow the chunk until it holds ~chunk_edges edges
        j = i + 1
        budget = int(rowptr[rows[i] + 1] - rowptr[rows[i]])
        while j < rows.numel() and budget < chunk_edges:
            budget += int(rowptr[rows[j] + 1] - rowptr[rows[j]])
            j += 1
        rr = rows[i:j]
        starts, ends = rowptr[rr], rowptr[rr + 1]
        lens = ends - starts
        local = torch.repeat_interleave(torch.arange(rr.numel()), lens)
        offs = torch.arange(int(lens.sum())) - torch.repeat_interleave(lens.cumsum(0) - lens, lens)
        k = torch.repeat_interleave(starts, lens) + offs
        src = col[k]
        e = asrc[src].double() + adst[rr][local].double()
        e = torch.where(e > 0, e, e * negative_slope)
        m = e.new_full((rr.numel(), H), float("-inf")).scatter_reduce(
            0, local.view(-1, 1).expand_as(e), e, "amax", include_self=True)
        p = (e - m[local]).exp()
        den = e.new_zeros((rr.numel(), H)).index_add_(0, local, p) + 1e-16
        a = p / den[local]
        msg = h[src].double().view(-1, H, C) * a.unsqueeze(-1)
        agg = msg.new_zeros((rr.numel(), H, C)).index_add_(0, local, msg)
        agg = agg.view(-1, H * C) if concat else agg.mean(dim=1)
        if bias is not None:
            agg = agg + bias.double()
        agg = _act(agg, act)
        if log_softmax:
            agg = F.log_softmax(agg, dim=-1)
        outs.append(agg)
        i = j
    return torch.cat(outs) if outs else torch.empty((0, Fw if concat else C), dtype=torch.float64)


def gat_layer_sample(x_rows, weight, att_src, att_dst, bias, heads, channels, h_src, asrc_src,
                     rowptr, col, negative_slope=0.2):
    """The CPU-baseline sample of one GAT layer: PyG's op sequence for the
    destination rows [0, R) (R = len(x_rows)), including those rows' share of
    the projection. h_src / asrc_src are the projected features of every
    source node (computed once, outside the timing) that the edges gather.

    Work per call = R rows of projection + the E_R = rowptr[R] edges of the
    edge chain (gat.1-raw-torch.mlir:5-129, restricted to the sample)."""
    H, C = heads, channels
    R = x_rows.size(0)
    h = (x_rows @ weight.t()).view(-1, H, C)  # this sample's share of aten.linear
    a_dst = (h * att_dst.view(1, H, C)).sum(dim=-1)
    e_r = int(rowptr[R])
    src = torch.as_tensor(col[:e_r], dtype=torch.int64)
    dst = torch.repeat_interleave(torch.arange(R), torch.as_tensor(rowptr[: R + 1]).diff())
    e = F.leaky_relu(asrc_src.index_select(0, src) + a_dst.index_select(0, dst), negative_slope)
    idx = dst.view(-1, 1).expand_as(e)
    m = e.new_zeros((R, H)).scatter_reduce(0, idx, e.detach(), "amax", include_self=False)
    p = (e - m.index_select(0, dst)).exp()
    s = e.new_zeros((R, H)).scatter_add(0, idx, p) + 1e-16
    alpha = p / s.index_select(0, dst)
    msg = alpha.unsqueeze(-1) * h_src.view(-1, H, C).index_select(0, src)
    out = h.new_zeros((R, H, C)).scatter_add(0, dst.view(-1, 1, 1).expand_as(msg), msg)
    out = out.view(-1, H * C)
    if bias is not None:
        out = out + bias
    return F.elu(out)


def gat_aggregate_sample(rowptr, col, h_src, asrc_src, adst_rows, heads, negative_slope=0.2):
    """The CPU-baseline sample of the fused chain alone (given h, a_src,
    a_dst; no projection, bias or activation): PyG's op sequence for the
    destination rows [0, R), R = len(adst_rows), over the edges
    col[:rowptr[R]] (gat.1-raw-torch.mlir:25-125)."""
    H = heads
    R = adst_rows.size(0)
    C = h_src.size(1) // H
    e_r = int(rowptr[R])
    src = torch.as_tensor(col[:e_r], dtype=torch.int64)
    dst = torch.repeat_interleave(torch.arange(R), torch.as_tensor(rowptr[: R + 1]).diff())
    e = F.leaky_relu(asrc_src.index_select(0, src) + adst_rows.index_select(0, dst), negative_slope)
    idx = dst.view(-1, 1).expand_as(e)
    m = e.new_zeros((R, H)).scatter_reduce(0, idx, e, "amax", include_self=False)
    p = (e - m.index_select(0, dst)).exp()
    s = e.new_zeros((R, H)).scatter_add(0, idx, p) + 1e-16
    alpha = p / s.index_select(0, dst)
    msg = alpha.unsqueeze(-1) * h_src.view(-1, H, C).index_select(0, src)
    out = h_src.new_zeros((R, H, C)).scatter_add(0, dst.view(-1, 1, 1).expand_as(msg), msg)
    return out.view(-1, H * C)


def gcn_rows_fp64(rowptr, col, w, h, *, rows=None, bias=None, act=None, log_softmax=False):
    """GCN aggregation of given h in float64 for destination rows `rows`."""
    rowptr = torch.as_tensor(rowptr, dtype=torch.int64)
    col = torch.as_tensor(col, dtype=torch.int64)
    n = rowptr.numel() - 1
    rows = torch.arange(n) if rows is None else torch.as_tensor(rows, dtype=torch.int64)
    starts, ends = rowptr[rows], rowptr[rows + 1]
    lens = ends - starts
    local = torch.repeat_interleave(torch.arange(rows.numel()), lens)
    offs = torch.arange(int(lens.sum())) - torch.repeat_interleave(lens.cumsum(0) - lens, lens)
    k = torch.repeat_interleave(starts, lens) + offs
    agg = h.new_zeros((rows.numel(), h.size(1)), dtype=torch.float64).index_add_(
        0, local, h[col[k]].double() * torch.as_tensor(w)[k].double()[:, None])
    if bias is not None:
        agg = agg + bias.double()
    agg = _act(agg, act)
    return F.log_softmax(agg, dim=-1) if log_softmax else agg


# ---------------------------------------------------------------------------
# Models (same layer order as gnnc/examples/models/{gcn,gat}.py)
# ---------------------------------------------------------------------------


def gcn_forward(model, x, crow, col, val):
    """Forward of the example GCN model on a pre-normalised CSR, from its parameters."""
    convs = [getattr(model, f"conv{i}") for i in range(1, model.num_layers + 1)]
    h = x.to(torch.float32)
    for i, conv in enumerate(convs):
        last = i == len(convs) - 1
        h = gcn_layer(h, crow, col, val, conv.lin.weight.detach(),
                      None if conv.bias is None else conv.bias.detach(),
                      act=None if last else "relu", log_softmax=last)
    return h


def sage_forward(model, x, crow, col, val):
    """Forward of the example SAGE model on a CSR adjacency, from its parameters."""
    convs = [getattr(model, f"conv{i}") for i in range(1, model.num_layers + 1)]
    h = x.to(torch.float32)
    for i, conv in enumerate(convs):
        last = i == len(convs) - 1
        h = sage_layer(h, crow, col, val, conv.lin_l.weight.detach(),
                       None if conv.lin_l.bias is None else conv.lin_l.bias.detach(),
                       conv.lin_r.weight.detach(), act=None if last else "relu",
                       log_softmax=last)
    return h


def gat_forward(model, x, edge_index):
    """Forward of the example GAT model, from its parameters."""
    convs = [getattr(model, f"conv{i}") for i in range(1, model.num_layers + 1)]
    h = x.to(torch.float32)
    for i, conv in enumerate(convs):
        last = i == len(convs) - 1
        h = gat_layer(h, edge_index, conv.lin.weight.detach(), conv.att_src.detach(),
                      conv.att_dst.detach(), None if conv.bias is None else conv.bias.detach(),
                      conv.heads, conv.out_channels, concat=conv.concat,
                      negative_slope=conv.negative_slope, add_self_loops=conv.add_self_loops,
                      act=None if last else "elu", log_softmax=last)
    return h


# ---------------------------------------------------------------------------
# Known-answer inputs defined by the reference's probe kernels
# ---------------------------------------------------------------------------


def kat_softmax_inputs():
    """alpha [64,64] CSR and X [64,32] of experiments/gat-gpu-codegen/gat-kernel.mlir:138-185.

    Stored pattern (i+j) % 11 == 0 with value ((i+2j) % 13 - 6) * 0.3f; the
    dense -> CSR sparse_tensor.convert stores nonzeros only, so the 29 pattern
    positions whose value is exactly 0 are not edges. X[j,k] = 0.01f*j + 0.001f*k."""
    i = np.arange(64)[:, None]
    j = np.arange(64)[None, :]
    val = (((i + 2 * j) % 13) - 6).astype(np.float32) * np.float32(0.3)
    mask = ((i + j) % 11 == 0) & (val != 0)
    crow = np.concatenate([[0], np.cumsum(mask.sum(1))]).astype(np.int64)
    rr, cc = np.nonzero(mask)
    x = (np.arange(64)[:, None].astype(np.float32) * np.float32(0.01)
         + np.arange(32)[None, :].astype(np.float32) * np.float32(0.001)).astype(np.float32)
    return crow, cc.astype(np.int64), val[rr, cc], x


def kat_spmm_inputs(which: str):
    """8x8 CSR A and dense B of experiments/sparsifier-coo-check/{01-spmm-csr,05-spmm-weighted-csr}.mlir."""
    i = np.arange(8)[:, None]
    j = np.arange(8)[None, :]
    s = (i + j).astype(np.float32)
    if which == "01":
        a = np.where((i + j) % 3 == 0, s, 0).astype(np.float32)
        b = (np.arange(64).reshape(8, 8).astype(np.float32) * np.float32(0.01)).astype(np.float32)
    else:
        a = np.where((i + j) % 3 == 0, s * np.float32(0.5), 0).astype(np.float32)
        b = (np.arange(8)[:, None] * 10 + np.arange(4)[None, :]).astype(np.float32)
    mask = a != 0
    crow = np.concatenate([[0], np.cumsum(mask.sum(1))]).astype(np.int64)
    rr, cc = np.nonzero(mask)
    return crow, cc.astype(np.int64), a[rr, cc], b
