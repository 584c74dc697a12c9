"""Aggregation kernels vs the oracle: GCN SpMM, fused GAT, softmax over given scores.

Covers the reference's known answers, the degree-skew paths (warp rows, CTA
rows, rows split across CTAs + merge), empty rows, odd widths, bf16 features,
mean-over-heads, fused activations / log_softmax and run-to-run determinism.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch
from conftest import GOLDEN
from gpu_util import assert_close, random_graph

from oracle import gnn_oracle as O

pytestmark = pytest.mark.gpu


def _plan(rowptr, cta=0, split=0):
    from gnnc.b200 import runtime as rt

    return rt.Plan(rowptr, cta_threshold=cta, split_threshold=split)


def _csr(device, crow, col):
    return (torch.as_tensor(np.asarray(crow), dtype=torch.int32, device=device),
            torch.as_tensor(np.asarray(col), dtype=torch.int32, device=device))


@pytest.mark.parametrize("which", ["01", "05"])
def test_spmm_known_answers(device, which):
    from gnnc.b200 import runtime as rt

    crow, col, val, b = O.kat_spmm_inputs(which)
    y = np.load(GOLDEN / "kat_spmm.npz")[f"y{which}"]
    rowptr, c = _csr(device, crow, col)
    w = torch.from_numpy(val).to(device)
    h = rt.empty_rows(b.shape[0], b.shape[1], torch.float32, device)
    h.copy_(torch.from_numpy(b))
    out = rt.gcn_aggregate(_plan(rowptr), rowptr, c, w, h)
    np.testing.assert_allclose(out.cpu().numpy(), y, rtol=1e-6, atol=1e-5)


@pytest.mark.parametrize("cta,split", [(0, 0), (2, 4)])
def test_softmax_spmm_known_answer(device, cta, split):
    """experiments/gat-gpu-codegen/dumps/cpu.out.txt through gnnc_softmax_aggregate (eps = 0)."""
    from gnnc.b200 import runtime as rt

    crow, col, val, x = O.kat_softmax_inputs()
    y = np.load(GOLDEN / "kat_softmax.npz")["y"]
    rowptr, c = _csr(device, crow, col)
    h = rt.empty_rows(64, 32, torch.float32, device)
    h.copy_(torch.from_numpy(x))
    s = torch.from_numpy(val).to(device).view(-1, 1)
    out = rt.softmax_aggregate(_plan(rowptr, cta, split), rowptr, c, s, h, heads=1, eps=0.0)
    np.testing.assert_allclose(out.cpu().numpy(), y, rtol=1e-5, atol=5e-6)


def _gcn_case(device, n, e, F, dtype, heavy, cta, split, act, lsm, seed):
    from gnnc.b200 import runtime as rt

    ei = random_graph(n, e, seed, heavy=heavy)
    rowptr, col, mult = rt.csr_from_coo(ei.to(device), n, self_loops=True, dedupe=True)
    _, _, w = rt.gcn_norm(rowptr, col, mult)
    g = torch.Generator().manual_seed(seed)
    h_host = torch.randn(n, F, generator=g).to(dtype)
    h = rt.empty_rows(n, F, dtype, device)
    h.copy_(h_host)
    bias = torch.randn(F, generator=g)
    out = rt.gcn_aggregate(_plan(rowptr, cta, split), rowptr, col, w, h, bias=bias.to(device),
                           act=act, log_softmax=lsm)
    ref = O.gcn_rows_fp64(rowptr.cpu(), col.cpu(), w.cpu(), h_host.double(), bias=bias,
                          act={0: None, 1: "relu", 2: "elu"}[act], log_softmax=lsm)
    return out, ref


@pytest.mark.parametrize(
    "n,e,F,dtype,heavy,cta,split",
    [
        (500, 4000, 7, torch.float32, (), 0, 0),
        (500, 4000, 47, torch.float32, ((3, 900),), 0, 0),
        (2000, 30000, 256, torch.float32, ((5, 9000), (9, 300)), 0, 0),
        (2000, 30000, 256, torch.bfloat16, ((5, 9000),), 0, 0),
        (3000, 20000, 64, torch.float32, ((1, 700), (2, 70)), 16, 64),
        (100, 300, 3, torch.float32, (), 1, 2),
        (700, 6000, 600, torch.float32, (), 0, 0),
    ],
)
def test_gcn_aggregate_matches_oracle(device, n, e, F, dtype, heavy, cta, split):
    out, ref = _gcn_case(device, n, e, F, dtype, heavy, cta, split, act=1, lsm=False, seed=n + F)
    assert_close(out, ref)


def test_gcn_aggregate_log_softmax_epilogue(device):
    out, ref = _gcn_case(device, 800, 8000, 47, torch.float32, ((0, 5000),), 0, 0, act=0,
                         lsm=True, seed=4)
    assert_close(out, ref)


def test_elu_keeps_relative_accuracy_near_zero(device):
    """ELU of small negative sums (|v| < 1e-3) is expm1(v) to a relative 1e-4
    with no absolute slack: exp(v) - 1 would cancel there."""
    from gnnc.b200 import runtime as rt

    n = 3000
    ei = random_graph(n, 30000, 17, heavy=((4, 2000),))
    rowptr, col, mult = rt.csr_from_coo(ei.to(device), n, self_loops=True, dedupe=True)
    _, _, w = rt.gcn_norm(rowptr, col, mult)
    g = torch.Generator().manual_seed(17)
    # strictly negative features: every row sum is negative and below 1e-3 in size
    h_host = -(torch.rand(n, 64, generator=g) * 5e-5 + 1e-8)
    h = rt.empty_rows(n, 64, torch.float32, device)
    h.copy_(h_host)
    out = rt.gcn_aggregate(_plan(rowptr), rowptr, col, w, h, act=rt.ACT_ELU).double().cpu()
    agg = O.gcn_rows_fp64(rowptr.cpu(), col.cpu(), w.cpu(), h_host.double())
    assert float(agg.abs().max()) < 1e-3 and bool((agg < 0).all())
    np.testing.assert_allclose(out.numpy(), torch.expm1(agg).numpy(), rtol=1e-4, atol=0)


def _gat_case(device, n, e, H, C, dtype, heavy, cta, split, concat, act, lsm, seed,
              self_loops=True, out_dtype=torch.float32, equal_logits=False):
    from gnnc.b200 import runtime as rt

    ei = random_graph(n, e, seed, heavy=heavy, loops=0 if not self_loops else 3)
    rowptr, col, _ = rt.csr_from_coo(ei.to(device), n, self_loops=self_loops, dedupe=False)
    g = torch.Generator().manual_seed(seed)
    h_host = torch.randn(n, H * C, generator=g).to(dtype)
    if equal_logits:
        asrc = torch.zeros(n, H)
        adst = torch.zeros(n, H)
    else:
        asrc = torch.randn(n, H, generator=g)
        adst = torch.randn(n, H, generator=g)
    bias = torch.randn(H * C if concat else C, generator=g)
    h = rt.empty_rows(n, H * C, dtype, device)
    h.copy_(h_host)
    out = rt.gat_aggregate(
        _plan(rowptr, cta, split), rowptr, col, h, asrc.to(device), adst.to(device), heads=H,
        concat=concat, bias=bias.to(device), act=act, log_softmax=lsm, out_dtype=out_dtype,
    )
    ref = O.gat_rows_fp64(rowptr.cpu(), col.cpu(), h_host.double(), asrc, adst, H, concat=concat,
                          bias=bias, act={0: None, 1: "relu", 2: "elu"}[act], log_softmax=lsm)
    return out, ref, rowptr


@pytest.mark.parametrize(
    "n,e,H,C,dtype,heavy,cta,split,concat",
    [
        (500, 5000, 1, 7, torch.float32, (), 0, 0, False),
        (500, 5000, 8, 8, torch.float32, ((3, 600),), 0, 0, True),
        (2000, 40000, 4, 64, torch.float32, ((5, 20000), (8, 3000)), 0, 0, True),
        (2000, 40000, 4, 64, torch.bfloat16, ((5, 20000), (8, 3000)), 0, 0, True),
        (1500, 20000, 4, 64, torch.bfloat16, ((1, 5000),), 32, 128, True),
        (900, 8000, 3, 5, torch.float32, ((2, 2000),), 8, 64, True),
        (900, 8000, 3, 5, torch.float32, ((2, 2000),), 8, 64, False),
        (1200, 9000, 1, 47, torch.float32, ((7, 4500),), 0, 0, False),
        (600, 6000, 16, 4, torch.float32, (), 0, 0, True),
        (400, 3000, 2, 128, torch.float32, ((0, 1000),), 0, 0, True),
    ],
)
def test_gat_aggregate_matches_oracle(device, n, e, H, C, dtype, heavy, cta, split, concat):
    out, ref, _ = _gat_case(device, n, e, H, C, dtype, heavy, cta, split, concat, act=2,
                            lsm=False, seed=n + H * C)
    assert_close(out, ref)


def test_gat_log_softmax_mean_epilogue(device):
    out, ref, _ = _gat_case(device, 1000, 9000, 4, 47, torch.float32, ((3, 6000),), 0, 0,
                            concat=False, act=0, lsm=True, seed=12)
    assert_close(out, ref)


def test_gat_empty_rows_without_self_loops(device):
    """Nodes with no incoming edge get bias only (PyG scatter_add of nothing)."""
    out, ref, rowptr = _gat_case(device, 3000, 1500, 2, 16, torch.float32, (), 0, 0, True, act=0,
                                 lsm=False, seed=21, self_loops=False)
    deg = rowptr.diff().cpu()
    assert int((deg == 0).sum()) > 1000
    assert_close(out, ref)


def test_gat_all_equal_logits_is_mean(device):
    out, ref, _ = _gat_case(device, 800, 6000, 4, 16, torch.float32, ((2, 5000),), 0, 0, True,
                            act=0, lsm=False, seed=3, equal_logits=True)
    assert_close(out, ref)


def test_gat_bf16_output_within_2e2(device):
    out, ref, _ = _gat_case(device, 1500, 20000, 4, 64, torch.bfloat16, ((9, 9000),), 0, 0, True,
                            act=2, lsm=False, seed=8, out_dtype=torch.bfloat16)
    assert_close(out, ref, rtol=2e-2, atol=2e-2)


def test_gat_deterministic_across_runs(device):
    from gnnc.b200 import runtime as rt

    n = 3000
    ei = random_graph(n, 60000, 5, heavy=((1, 15000), (2, 2500)))
    rowptr, col, _ = rt.csr_from_coo(ei.to(device), n, self_loops=True, dedupe=False)
    plan = _plan(rowptr)
    assert plan.info()["n_split_rows"] == 1 and plan.info()["n_cta_rows"] >= 1
    h = torch.randn(n, 256, device=device).to(torch.bfloat16)
    asrc = torch.randn(n, 4, device=device)
    adst = torch.randn(n, 4, device=device)
    a = rt.gat_aggregate(plan, rowptr, col, h, asrc, adst, heads=4)
    b = rt.gat_aggregate(plan, rowptr, col, h, asrc, adst, heads=4)
    assert torch.equal(a.view(torch.int32), b.view(torch.int32))


def test_bad_column_is_skipped_and_reported(device):
    """A column index past the feature table is never dereferenced; the kernel
    flags it and gnnc_synchronize reports GNNC_ERR_BOUNDS."""
    from gnnc.b200 import runtime as rt
    from gnnc.b200._lib import GnncInvalidArgument

    rowptr = torch.tensor([0, 2, 3], dtype=torch.int32, device=device)
    col = torch.tensor([0, 1, 1000], dtype=torch.int32, device=device)
    w = torch.ones(3, device=device)
    h = torch.ones(4, 8, device=device)
    rt.gcn_aggregate(_plan(rowptr), rowptr, col, w, h)
    with pytest.raises(GnncInvalidArgument):
        rt.Context.get(device).synchronize()
    rt.Context.get(device).synchronize()  # flag cleared


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("H,C,concat", [(1, 256, True), (2, 128, True), (8, 32, True),
                                         (4, 64, False), (3, 256, True)])
def test_gat_256_wide_head_counts(device, H, C, concat, dtype):
    """Rows of 256 features (bf16: one 16-byte load per lane; fp32: two) for
    every head count the compile-time edge loops cover, a mean-over-heads
    epilogue, and a width that takes the generic loop (3 x 256 features)."""
    out, ref, _ = _gat_case(device, 1800, 30000, H, C, dtype, ((4, 7000), (6, 900)), 0,
                            0, concat, act=2, lsm=False, seed=40 + H)
    assert_close(out, ref)


def test_softmax_aggregate_bf16_256_wide(device):
    """Given scores [E, 4] with bf16 256-wide rows (the score-row vector loads,
    including the lanes past a chunk's last edge)."""
    from gnnc.b200 import runtime as rt

    n, H = 1700, 4
    ei = random_graph(n, 25000, 77, heavy=((3, 6000),))
    rowptr, col, _ = rt.csr_from_coo(ei.to(device), n, self_loops=True, dedupe=False)
    E = col.numel()
    g = torch.Generator().manual_seed(77)
    s = torch.randn(E, H, generator=g)
    h_host = torch.randn(n, 256, generator=g).to(torch.bfloat16)
    h = rt.empty_rows(n, 256, torch.bfloat16, device)
    h.copy_(h_host)
    out = rt.softmax_aggregate(_plan(rowptr), rowptr, col, s.to(device), h, heads=H)
    rp, c = rowptr.cpu().long(), col.cpu().long()
    hd64 = h_host.double()
    ref = torch.cat([O.softmax_aggregate(rp, c, s[:, k].double(), hd64[:, 64 * k : 64 * k + 64],
                                         eps=1e-16) for k in range(H)], dim=1)
    assert_close(out, ref)


def test_bad_column_bf16_256_wide(device):
    from gnnc.b200 import runtime as rt
    from gnnc.b200._lib import GnncInvalidArgument

    rowptr = torch.tensor([0, 2, 5], dtype=torch.int32, device=device)
    col = torch.tensor([0, 1, 1, 7, 1 << 30], dtype=torch.int32, device=device)
    h = torch.ones(4, 256, device=device).to(torch.bfloat16)
    asrc = torch.zeros(4, 4, device=device)
    adst = torch.zeros(2, 4, device=device)
    out = rt.gat_aggregate(_plan(rowptr), rowptr, col, h, asrc, adst, heads=4)
    with pytest.raises(GnncInvalidArgument):
        rt.Context.get(device).synchronize()
    # the bad edges are dropped: row 1 keeps its one in-range edge
    assert torch.allclose(out.cpu(), torch.ones(2, 256))


@pytest.mark.parametrize("H,C,concat,act,lsm", [(1, 47, False, 0, True), (8, 8, True, 2, False),
                                                (2, 24, False, 1, False), (4, 16, True, 0, True),
                                                (1, 40, True, 2, True)])
def test_gat_bf16_narrow_rows(device, H, C, concat, act, lsm):
    """bf16 rows of 33-64 features (four edges side by side per warp), every
    compile-time head count, both head reductions and the log_softmax epilogue
    (the last c4 layer is 1 x 47, mean, log_softmax)."""
    out, ref, _ = _gat_case(device, 1800, 30000, H, C, torch.bfloat16, ((4, 7000), (6, 900)), 0,
                            0, concat, act=act, lsm=lsm, seed=60 + H * C)
    assert_close(out, ref)


@pytest.mark.parametrize("F,lsm", [(47, True), (64, False), (40, False)])
def test_gcn_bf16_narrow_rows(device, F, lsm):
    out, ref = _gcn_case(device, 2500, 30000, F, torch.bfloat16, ((5, 9000), (9, 300)), 0, 0,
                         act=0 if lsm else 1, lsm=lsm, seed=F)
    assert_close(out, ref)


def test_softmax_aggregate_bf16_narrow(device):
    from gnnc.b200 import runtime as rt

    n = 1200
    ei = random_graph(n, 15000, 91, heavy=((2, 5000),))
    rowptr, col, _ = rt.csr_from_coo(ei.to(device), n, self_loops=True, dedupe=False)
    g = torch.Generator().manual_seed(91)
    s = torch.randn(col.numel(), generator=g)
    h_host = torch.randn(n, 48, generator=g).to(torch.bfloat16)
    h = rt.empty_rows(n, 48, torch.bfloat16, device)
    h.copy_(h_host)
    out = rt.softmax_aggregate(_plan(rowptr), rowptr, col, s.to(device), h, heads=1)
    ref = O.softmax_aggregate(rowptr.cpu().long(), col.cpu().long(), s.double(), h_host.double(),
                              eps=1e-16)
    assert_close(out, ref)



def test_mean_norm_is_bit_exact(device):
    """gnnc_mean_norm: value / max(count of nonzero values in the row, 1), IEEE
    division; zero values stay zero and do not count; empty rows are fine."""
    from gnnc.b200 import runtime as rt

    n = 3000
    ei = random_graph(n, 40000, 17, heavy=((3, 5000),))
    rowptr, col, _ = rt.csr_from_coo(ei.to(device), n, self_loops=False, dedupe=False)
    g = torch.Generator().manual_seed(17)
    val = torch.rand(col.numel(), generator=g)
    val[torch.rand(col.numel(), generator=g) < 0.2] = 0.0
    w = rt.mean_norm(rowptr, val.to(device)).cpu()
    assert torch.equal(w, O.mean_weights(rowptr.cpu(), val))
    w1 = rt.mean_norm(rowptr).cpu()
    assert torch.equal(w1, O.mean_weights(rowptr.cpu()))


@pytest.mark.parametrize(
    "F,dtype,act,lsm,cta,split",
    [(7, torch.float32, 1, False, 0, 0), (47, torch.bfloat16, 0, True, 0, 0),
     (256, torch.bfloat16, 1, False, 0, 0), (256, torch.float32, 2, False, 16, 64),
     (600, torch.float32, 1, False, 0, 0)],
)
def test_sage_aggregate_matches_oracle(device, F, dtype, act, lsm, cta, split):
    """out = A_mean . h + root + bias (then act / log_softmax) over warp, CTA and
    split rows, with the root term in both epilogues."""
    from gnnc.b200 import runtime as rt

    n = 2500
    ei = random_graph(n, 30000, F, heavy=((5, 9000), (9, 300)))
    rowptr, col, mult = rt.csr_from_coo(ei.to(device), n, self_loops=True, dedupe=True)
    _, _, wn = rt.gcn_norm(rowptr, col, mult)
    w = rt.mean_norm(rowptr, wn)
    g = torch.Generator().manual_seed(F)
    h_host = torch.randn(n, F, generator=g).to(dtype)
    root_host = torch.randn(n, F, generator=g).to(dtype)
    h = rt.empty_rows(n, F, dtype, device)
    h.copy_(h_host)
    root = rt.empty_rows(n, F, dtype, device)
    root.copy_(root_host)
    bias = torch.randn(F, generator=g)
    out = rt.sage_aggregate(_plan(rowptr, cta, split), rowptr, col, w, h, root,
                            bias=bias.to(device), act=act, log_softmax=lsm)
    agg = O.spmm_csr(rowptr.cpu(), col.cpu(), w.cpu().double(), h_host.double())
    ref = agg + root_host.double() + bias.double()
    ref = {0: ref, 1: torch.relu(ref), 2: torch.nn.functional.elu(ref)}[act]
    if lsm:
        ref = torch.log_softmax(ref, dim=-1)
    assert_close(out, ref)


def test_partition_plans_split_like_the_whole_graph(device):
    """A rank's plan given whole_graph_split_threshold splits exactly the rows
    the single-GPU plan splits, so its output rows equal the single-GPU rows
    bit for bit (its own default follows its smaller edge count and may split
    rows the single-GPU plan keeps whole)."""
    from gnnc.b200 import partition as P
    from gnnc.b200 import runtime as rt

    g = torch.Generator().manual_seed(11)
    n = 100_000
    deg = torch.randint(20, 80, (n,), generator=g)
    hubs = torch.randperm(n, generator=g)[:40]
    deg[hubs] = torch.randint(4200, 9000, (40,), generator=g)  # between the two thresholds
    rowptr = torch.zeros(n + 1, dtype=torch.int64)
    rowptr[1:] = deg.cumsum(0)
    E = int(rowptr[-1])
    col = torch.randint(0, n, (E,), generator=g, dtype=torch.int32)
    rowptr_d, col_d = rowptr.to(torch.int32).to(device), col.to(device)
    h = torch.randn(n, 256, generator=g).to(torch.bfloat16).to(device)
    a = (torch.randn(n, 4, generator=g) * 0.5).to(device)
    d = (torch.randn(n, 4, generator=g) * 0.5).to(device)
    sms = torch.cuda.get_device_properties(device).multi_processor_count
    thr = P.whole_graph_split_threshold(E, sms)
    assert thr > 4096  # the graph is large enough for the adaptive default
    whole = rt.Plan(rowptr_d)
    assert whole.info() == rt.Plan(rowptr_d, split_threshold=thr).info()
    kw = dict(heads=4, concat=True, act=rt.ACT_ELU, out_dtype=torch.bfloat16)
    full = rt.gat_aggregate(whole, rowptr_d, col_d, h, a, d, **kw)
    for r in range(4):
        rr = P.row_range(n, 4, r)
        rp_l, col_l = P.local_csr(rowptr_d, col_d, rr)
        plan = rt.Plan(rp_l, split_threshold=thr)
        assert plan.info()["n_split_rows"] == int((deg[rr.begin : rr.end] > thr).sum())
        out = rt.gat_aggregate(plan, rp_l, col_l, h, a, d[rr.begin : rr.end], **kw)
        assert torch.equal(out, full[rr.begin : rr.end]), f"rank {r}"


def test_host_row_chunks_split_like_the_whole_graph(device):
    """The row chunks a host-bound result is aggregated in (DeviceGraph.row_chunks)
    split exactly the rows the whole graph's plan splits, so the chunked rows
    equal the single launch bit for bit; a chunk's own default threshold
    follows its smaller edge count and would split hub rows the whole plan
    keeps whole."""
    from gnnc.b200 import partition as P
    from gnnc.b200 import runtime as rt
    from gnnc.b200.program import DeviceGraph

    g = torch.Generator().manual_seed(12)
    n = 100_000
    deg = torch.randint(20, 80, (n,), generator=g)
    hubs = torch.randperm(n, generator=g)[:40]
    deg[hubs] = torch.randint(4200, 9000, (40,), generator=g)
    rowptr = torch.zeros(n + 1, dtype=torch.int64)
    rowptr[1:] = deg.cumsum(0)
    E = int(rowptr[-1])
    col = torch.randint(0, n, (E,), generator=g, dtype=torch.int32)
    rowptr_d, col_d = rowptr.to(torch.int32).to(device), col.to(device)
    h = torch.randn(n, 256, generator=g).to(torch.bfloat16).to(device)
    a = (torch.randn(n, 4, generator=g) * 0.5).to(device)
    d = (torch.randn(n, 4, generator=g) * 0.5).to(device)
    sms = torch.cuda.get_device_properties(device).multi_processor_count
    thr = P.whole_graph_split_threshold(E, sms)
    k = 8
    # some hub rows lie between a chunk's own default and the whole graph's threshold
    assert int(((deg > P.whole_graph_split_threshold(E // k, sms)) & (deg <= thr)).sum()) > 0
    dg = DeviceGraph(rowptr_d, col_d, None, rt.Plan(rowptr_d), n)
    whole = dg.plan.info()
    assert whole["n_split_rows"] == int((deg > thr).sum())
    chunks = dg.row_chunks(k)
    assert len(chunks) == k
    assert sum(p.info()["n_split_rows"] for _, _, p in chunks) == whole["n_split_rows"]
    kw = dict(heads=4, concat=True, act=rt.ACT_ELU, out_dtype=torch.bfloat16)
    full = rt.gat_aggregate(dg.plan, rowptr_d, col_d, h, a, d, **kw)
    out = torch.empty_like(full)
    for r0, r1, plan in chunks:
        rt.gat_aggregate(plan, rowptr_d[r0 : r1 + 1], col_d, h, a, d[r0:r1], out=out[r0:r1], **kw)
    assert torch.equal(out, full)


@pytest.mark.parametrize("heads", [4, 0])
def test_edge_stream_with_empty_rows_hubs_and_splits(device, heads):
    """The prefetched edge stream (256-wide bf16 rows, GAT and GCN modes) over
    runs of rows without edges (inside tasks, at task starts and ends), hub
    rows the plan gives to the CTA path (which cut the stream tasks) and rows
    split across CTAs, against the oracle."""
    from gnnc.b200 import runtime as rt

    n = 20_000
    g = torch.Generator().manual_seed(77)
    # sources 0..n-1, destinations only in the first ~60 % of rows and a few hubs
    dst = torch.randint(0, int(n * 0.6), (90_000,), generator=g)
    src = torch.randint(0, n, (90_000,), generator=g)
    hubs = [(n - 3, 6000), (n // 2, 2500), (100, 1500)]
    parts = [torch.stack([src, dst])]
    for node, deg in hubs:
        parts.append(torch.stack([torch.randint(0, n, (deg,), generator=g),
                                  torch.full((deg,), node)]))
    ei = torch.cat(parts, 1)
    rowptr, col, mult = rt.csr_from_coo(ei.to(device), n, self_loops=False, dedupe=heads == 0)
    deg = rowptr.diff().cpu()
    assert int((deg == 0).sum()) > 5000 and int(deg.max()) > 4096
    plan = rt.Plan(rowptr, cta_threshold=0, split_threshold=4096)
    assert plan.info()["n_split_rows"] >= 1
    F = 256
    h_host = torch.randn(n, F, generator=g).to(torch.bfloat16)
    h = rt.empty_rows(n, F, torch.bfloat16, device)
    h.copy_(h_host)
    bias = torch.randn(F, generator=g)
    if heads:
        asrc = torch.randn(n, heads, generator=g)
        adst = torch.randn(n, heads, generator=g)
        out = rt.gat_aggregate(plan, rowptr, col, h, asrc.to(device), adst.to(device), heads=heads,
                               bias=bias.to(device), act=rt.ACT_ELU, out_dtype=torch.bfloat16)
        ref = O.gat_rows_fp64(rowptr.cpu(), col.cpu(), h_host.double(), asrc, adst, heads,
                              bias=bias, act="elu")
    else:
        w = torch.rand(col.numel(), generator=g).to(device)
        out = rt.gcn_aggregate(plan, rowptr, col, w, h, bias=bias.to(device), act=rt.ACT_RELU,
                               out_dtype=torch.bfloat16)
        ref = O.gcn_rows_fp64(rowptr.cpu(), col.cpu(), w.cpu(), h_host.double(), bias=bias,
                              act="relu")
    assert_close(out, ref, rtol=2e-2, atol=2e-2)
    empty = deg == 0
    expect = torch.nn.functional.elu(bias) if heads else torch.relu(bias)
    assert torch.allclose(out.float().cpu()[empty], expect.expand(int(empty.sum()), F),
                          rtol=1e-2, atol=1e-2)
