"""Row-sampled parity at full graph sizes (TEST INFRASTRUCTURE ONLY).

The checker for graphs too large for the whole-graph oracle: the GPU output of
a layer is compared, on a set of destination rows, with the oracle's float64
restatement of the same layer computed from the same inputs. Importable only by
tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg; the product
path never calls it.

Rows checked: every row whose in-degree (self-loop included) exceeds a cut-off
(the hub rows that take the CTA and split-row paths of the kernels) plus a
seeded uniform sample of the other rows.

The layer restatements follow the reference's semantics exactly as
gnn_oracle.py does (GATConv: experiments/gatconv/dumps/gat.1-raw-torch.mlir:5-129;
GCNConv on a normalised CSR: test/reference/gcn.raw.mlir:6-21), restricted to
the sampled rows: only the sampled rows' edges and the rows they read are
projected.
"""

from __future__ import annotations

import warnings

import numpy as np
import torch
import torch.nn.functional as F

from oracle import gnn_oracle as O

warnings.filterwarnings("ignore", message=r".*Sparse CSR tensor support is in beta.*")
warnings.filterwarnings("ignore", message=r".*Sparse invariant checks are implicitly disabled.*")


def sample_rows(rowptr, *, sample: int, hub_degree: int, seed: int, extra=()) -> torch.Tensor:
    """Sorted unique int64 row ids: rows of degree > hub_degree, `extra`, and
    `sample` further rows drawn uniformly without replacement (seeded)."""
    rowptr = torch.as_tensor(rowptr, dtype=torch.int64).cpu()
    n = rowptr.numel() - 1
    deg = rowptr.diff()
    hubs = torch.nonzero(deg > hub_degree).flatten()
    rng = np.random.default_rng(seed)
    k = min(sample, n)
    drawn = torch.from_numpy(rng.choice(n, size=k, replace=False).astype(np.int64))
    ex = torch.as_tensor(list(extra), dtype=torch.int64)
    return torch.unique(torch.cat([hubs, drawn, ex]))


def csr_by_destination(edge_index: torch.Tensor, num_nodes: int):
    """(rowptr, col) int64 of edge_index [2, E] by destination, sources
    ascending within a row, with GATConv's self-loop handling (every (i, i)
    edge dropped, one loop per node added), sorted with torch on the host."""
    n = num_nodes
    keep = edge_index[0] != edge_index[1]
    loops = torch.arange(n, dtype=torch.int64)
    src = torch.cat([edge_index[0][keep], loops])
    dst = torch.cat([edge_index[1][keep], loops])
    key = torch.sort(dst * n + src).values
    rowptr = torch.zeros(n + 1, dtype=torch.int64)
    rowptr[1:] = torch.cumsum(torch.bincount(key // n, minlength=n), 0)
    return rowptr, key % n


def row_edges(rowptr, col, rows):
    """The edges of destination `rows` as a row-local CSR: (local rowptr over
    `rows`, global source id of every edge, each edge's index in `col`)."""
    rowptr = torch.as_tensor(rowptr, dtype=torch.int64)
    starts, ends = rowptr[rows], rowptr[rows + 1]
    lens = ends - starts
    offs = torch.arange(int(lens.sum())) - torch.repeat_interleave(lens.cumsum(0) - lens, lens)
    k = torch.repeat_interleave(starts, lens) + offs
    local = torch.zeros(rows.numel() + 1, dtype=torch.int64)
    local[1:] = lens.cumsum(0)
    src = torch.as_tensor(col, dtype=torch.int64)[k]
    return local, src, k


def _project(x_rows: torch.Tensor, weight: torch.Tensor, chunk: int = 1 << 18) -> torch.Tensor:
    """x_rows @ weight^T in float64 (x's stored values exactly), row chunk by row chunk."""
    wt = weight.double().t().contiguous()
    out = torch.empty((x_rows.size(0), wt.size(1)), dtype=torch.float64)
    for i in range(0, x_rows.size(0), chunk):
        torch.mm(x_rows[i : i + chunk].double(), wt, out=out[i : i + chunk])
    return out


def _weighted_rows(local, inv, vals, h_u) -> torch.Tensor:
    """out[r] = sum over row r's edges k of vals[k] * h_u[inv[k]] in float64,
    as one sparse (CSR) x dense product: the weighted scatter-add of messages
    without materialising the [E, F] message tensor."""
    a = torch.sparse_csr_tensor(local, inv, vals.double().contiguous(),
                                size=(local.numel() - 1, h_u.size(0)))
    return a @ h_u


def gat_rows_given_fp64(local, inv, h_u, a_s, a_d, heads: int, *, negative_slope=0.2,
                        concat=True, bias=None, act=None, log_softmax=False):
    """The GAT edge chain in float64 on a row-local CSR (local rowptr over the
    checked rows, inv = each edge's source as a row of h_u / a_s), op by op as
    gat.1-raw-torch.mlir:25-129: e = leaky_relu(a_src[src] + a_dst[dst]);
    m = row amax of e (include_self = False); p = exp(e - m); S = row sum of
    p + 1e-16; out = sum p / S * h[src]; then concat or mean over heads, bias,
    activation, log_softmax."""
    H = heads
    C = h_u.size(1) // H
    R = local.numel() - 1
    row = torch.repeat_interleave(torch.arange(R), local.diff())
    e = a_s.double()[inv] + a_d.double()[row]
    e = torch.where(e > 0, e, e * negative_slope)
    idx = row.view(-1, 1).expand_as(e)
    m = e.new_zeros((R, H)).scatter_reduce(0, idx, e, "amax", include_self=False)
    p = (e - m[row]).exp()
    den = e.new_zeros((R, H)).scatter_add(0, idx, p) + 1e-16
    alpha = p / den[row]
    hd = h_u.double()
    out = torch.cat([_weighted_rows(local, inv, alpha[:, k], hd[:, k * C : (k + 1) * C].contiguous())
                     for k in range(H)], dim=1)
    out = out if concat else out.view(R, H, C).mean(dim=1)
    if bias is not None:
        out = out + bias.double()
    out = O._act(out, act)
    return F.log_softmax(out, dim=-1) if log_softmax else out


def gat_conv_rows_fp64(x, rowptr, col, rows, weight, att_src, att_dst, bias, heads: int, *,
                       concat=True, negative_slope=0.2, act=None, log_softmax=False):
    """One GATConv layer (projection, attention coefficients, SDDMM, LeakyReLU,
    edge softmax, SpMM, heads, bias, activation) in float64 for destination
    `rows` of a CSR by destination that already holds its self-loops.

    x: [N, K] layer input (any float dtype; the exact stored values are used).
    Only the sources the rows' edges read, and the rows themselves, are
    projected. Returns [len(rows), F_out] float64."""
    rows = torch.as_tensor(rows, dtype=torch.int64)
    H = heads
    C = weight.size(0) // H
    local, src, _ = row_edges(rowptr, col, rows)
    uniq, inv = torch.unique(src, return_inverse=True)
    h_u = _project(x[uniq], weight)  # gat.1-raw-torch.mlir:5-10
    a_s = torch.einsum("uhc,hc->uh", h_u.view(-1, H, C), att_src.double().view(H, C))  # :11-17
    h_r = _project(x[rows], weight)
    a_d = torch.einsum("uhc,hc->uh", h_r.view(-1, H, C), att_dst.double().view(H, C))  # :18-24
    return gat_rows_given_fp64(local, inv, h_u, a_s, a_d, H, negative_slope=negative_slope,
                               concat=concat, bias=bias, act=act, log_softmax=log_softmax)


def gcn_conv_rows_fp64(x, rowptr, col, w, rows, weight, bias, *, act=None, log_softmax=False):
    """One GCNConv layer on a normalised CSR (linear without bias, weighted
    SpMM, + bias, activation) in float64 for destination `rows`
    (test/reference/gcn.raw.mlir:6-10)."""
    rows = torch.as_tensor(rows, dtype=torch.int64)
    local, src, k = row_edges(rowptr, col, rows)
    uniq, inv = torch.unique(src, return_inverse=True)
    h_u = _project(x[uniq], weight)
    out = _weighted_rows(local, inv, torch.as_tensor(w)[k], h_u)
    if bias is not None:
        out = out + bias.double()
    out = O._act(out, act)
    return F.log_softmax(out, dim=-1) if log_softmax else out


def compare(got: torch.Tensor, ref: torch.Tensor, *, rtol: float, atol: float) -> dict:
    """Elementwise |got - ref| <= atol + rtol * |ref| over the checked rows.

    Returns the verdict and the figures behind it: max abs error, max relative
    error over elements with |ref| >= 0.1 (smaller ones are bounded by atol),
    and the worst ratio |err| / (atol + rtol |ref|) (pass means <= 1)."""
    got = got.double()
    ref = ref.double()
    err = (got - ref).abs()
    bound = atol + rtol * ref.abs()
    big = ref.abs() >= 0.1
    finite = bool(torch.isfinite(got).all())
    return {
        "pass": finite and bool((err <= bound).all()),
        "max_abs_err": float(err.max()) if err.numel() else 0.0,
        "max_rel_err": float((err[big] / ref.abs()[big]).max()) if bool(big.any()) else 0.0,
        "worst_ratio_to_bound": float((err / bound).max()) if err.numel() else 0.0,
        "rtol": rtol,
        "atol": atol,
        "elements": int(err.numel()),
    }


def argmax_agreement(got: torch.Tensor, ref: torch.Tensor, max_abs_err: float) -> dict:
    """Class predictions of got vs ref over the checked rows.

    A prediction can differ only where the oracle's top-2 margin is at most
    twice the error of the two entries, so rows with margin <= 2 x the
    observed max abs error are near-ties (counted, not required to agree);
    every other row must agree ("pass"). Also reported: how many rows differ
    at all, and the largest oracle margin among them (how close the flips
    were)."""
    top2 = ref.double().topk(2, dim=1).values
    margin = top2[:, 0] - top2[:, 1]
    tie = margin <= 2 * max_abs_err
    differ = got.argmax(1) != ref.argmax(1)
    return {
        "pass": not bool((differ & ~tie).any()),
        "rows": int(got.size(0)),
        "disagree": int(differ.sum()),
        "disagree_decided": int((differ & ~tie).sum()),
        "near_ties": int(tie.sum()),
        "max_margin_of_disagreeing_rows": float(margin[differ].max()) if bool(differ.any()) else 0.0,
        "median_margin": float(margin.median()),
    }
