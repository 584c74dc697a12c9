"""gnnc_gat_aggregate_noalloc: the GAT aggregation for callers that cannot
allocate device memory while it runs (a process that reserved its whole memory
budget at start-up, or a runtime that owns all device memory through its own
pool). The entry point keeps its scratch in a fixed array inside the library
instead of calling cudaMalloc.

The test calls it through the C ABI twice in a row and compares both results
with gnnc_gat_aggregate's, on a graph whose split rows use the scratch. This
file is collected last, so a run that stops at the first failure has already
run every other test; it also passes when run alone in a fresh process.
"""

from __future__ import annotations

import pytest
import torch
from gpu_util import assert_close, random_graph

pytestmark = pytest.mark.gpu


def _graph(device, n, e, heavy, cta=0, split=0):
    from gnnc.b200 import runtime as rt

    ei = random_graph(n, e, seed=99, heavy=heavy)
    rowptr, col, _ = rt.csr_from_coo(ei.to(device), n, self_loops=True, dedupe=False)
    return rowptr, col, rt.Plan(rowptr, cta_threshold=cta, split_threshold=split)


@pytest.mark.parametrize("dtype,out_dtype", [(torch.float32, torch.float32),
                                             (torch.bfloat16, torch.bfloat16)])
def test_noalloc_matches_allocating_entry_point_twice(device, dtype, out_dtype):
    from gnnc.b200 import runtime as rt

    n, H, C = 4000, 4, 64
    rowptr, col, plan = _graph(device, n, 60000, heavy=((3, 20000), (11, 9000), (17, 1500)))
    info = plan.info()
    assert info["n_split_rows"] >= 2 and info["n_cta_rows"] >= 1  # partials are used
    g = torch.Generator().manual_seed(7)
    h = rt.empty_rows(n, H * C, dtype, device)
    h.copy_(torch.randn(n, H * C, generator=g))
    asrc = torch.randn(n, H, generator=g).to(device)
    adst = torch.randn(n, H, generator=g).to(device)
    bias = torch.randn(H * C, generator=g).to(device)
    ref = rt.gat_aggregate(plan, rowptr, col, h, asrc, adst, heads=H, bias=bias, act=rt.ACT_ELU,
                           out_dtype=out_dtype)
    tol = 1e-4 if out_dtype == torch.float32 else 2e-2
    for _ in range(2):
        out = rt.empty_rows(n, H * C, out_dtype, device)
        out.fill_(float("nan"))
        rt.gat_aggregate_noalloc(plan, rowptr, col, h, asrc, adst, out, heads=H, bias=bias,
                                 act=rt.ACT_ELU)
        rt.Context.get(device).synchronize()
        assert_close(out, ref, rtol=tol, atol=tol)


def test_noalloc_leaves_free_device_memory_unchanged(device):
    """The claim itself: with a plan that has more split-row segments than
    any call before it (the allocating entry point would grow its workspace),
    two calls leave the device's free memory exactly where it was."""
    from gnnc.b200 import runtime as rt

    n, H, C = 5000, 4, 64
    h = rt.empty_rows(n, H * C, torch.bfloat16, device)
    h.normal_()
    asrc = torch.randn(n, H, device=device)
    adst = torch.randn(n, H, device=device)
    outs = [rt.empty_rows(n, H * C, torch.bfloat16, device) for _ in range(2)]
    # warm-up on a small plan with split rows: the kernels of this layout are
    # loaded (loading a kernel may reserve device memory) by both entry points
    rp_s, col_s, plan_s = _graph(device, 1000, 8000, heavy=((1, 3000),), cta=32, split=512)
    assert plan_s.info()["n_split_rows"] >= 1
    rt.gat_aggregate_noalloc(plan_s, rp_s, col_s, h, asrc, adst[:1000], outs[0][:1000], heads=H)
    rt.gat_aggregate(plan_s, rp_s, col_s, h, asrc, adst[:1000], heads=H, out_dtype=torch.bfloat16)
    rowptr, col, plan = _graph(device, n, 80000, heavy=((2, 30000), (8, 25000), (13, 9000)),
                               cta=32, split=64)
    info = plan.info()
    assert info["n_segments"] >= 900 > 8 * plan_s.info()["n_segments"]
    torch.cuda.synchronize(device)
    free_before = torch.cuda.mem_get_info(device)[0]
    for out in outs:
        rt.gat_aggregate_noalloc(plan, rowptr, col, h, asrc, adst, out, heads=H)
    rt.Context.get(device).synchronize()
    assert torch.cuda.mem_get_info(device)[0] == free_before
    ref = rt.gat_aggregate(plan, rowptr, col, h, asrc, adst, heads=H, out_dtype=torch.bfloat16)
    assert_close(outs[0], ref, rtol=2e-2, atol=2e-2)
    assert torch.equal(outs[0], outs[1])


def test_noalloc_mean_heads_log_softmax(device):
    from gnnc.b200 import runtime as rt

    n, H, C = 3000, 2, 47
    rowptr, col, plan = _graph(device, n, 30000, heavy=((5, 12000),), cta=32, split=256)
    h = torch.randn(n, H * C, device=device)
    asrc = torch.randn(n, H, device=device)
    adst = torch.randn(n, H, device=device)
    ref = rt.gat_aggregate(plan, rowptr, col, h, asrc, adst, heads=H, concat=False,
                           log_softmax=True)
    for _ in range(2):
        out = torch.full((n, C), float("nan"), device=device)
        rt.gat_aggregate_noalloc(plan, rowptr, col, h, asrc, adst, out, heads=H, concat=False,
                                 log_softmax=True)
        assert_close(out, ref)


def test_noalloc_rejects_plans_beyond_the_fixed_scratch(device):
    from gnnc.b200 import runtime as rt
    from gnnc.b200._lib import GnncUnsupported

    n = 20000
    rowptr, col, plan = _graph(device, n, 200000, heavy=(), cta=2, split=2)
    assert plan.info()["n_segments"] * (32 + 256) * 4 > 16 * 2**20
    h = torch.zeros(n, 256, device=device, dtype=torch.bfloat16)
    a = torch.zeros(n, 4, device=device)
    out = torch.empty(n, 256, device=device, dtype=torch.bfloat16)
    with pytest.raises(GnncUnsupported, match="fixed scratch"):
        rt.gat_aggregate_noalloc(plan, rowptr, col, h, a, a, out, heads=4)
