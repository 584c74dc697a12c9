"""Dense projection (and GAT attention coefficients) vs a float64 reference."""

from __future__ import annotations

import pytest
import torch
from gpu_util import assert_close

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize(
    "n,k,f,heads,dtype",
    [
        (2708, 1433, 16, 1, torch.float32),
        (2708, 1433, 64, 8, torch.float32),
        (1000, 64, 7, 1, torch.float32),
        (5000, 128, 256, 4, torch.float32),
        (5000, 100, 256, 4, torch.bfloat16),
        (3001, 256, 48, 1, torch.bfloat16),
        (777, 256, 256, 4, torch.bfloat16),
        (129, 13, 5, 1, torch.float32),
    ],
)
def test_proj_matches_fp64(device, n, k, f, heads, dtype):
    from gnnc.b200 import runtime as rt

    g = torch.Generator().manual_seed(n + k + f)
    x = torch.randn(n, k, generator=g).to(dtype)
    w = (torch.randn(f, k, generator=g) / k**0.5).to(dtype)
    att_s = torch.randn(f, generator=g)
    att_d = torch.randn(f, generator=g)
    xd = rt.empty_rows(n, k, dtype, device)
    xd.copy_(x)
    wd = rt.empty_rows(f, k, dtype, device)
    wd.copy_(w)
    h, asrc, adst = rt.proj(xd, wd, att_src=att_s.to(device), att_dst=att_d.to(device),
                            heads=heads, out_dtype=torch.float32)
    ref = x.double() @ w.double().t()
    assert_close(h, ref, rtol=1e-4, atol=1e-4)
    C = f // heads
    rs = (ref.view(n, heads, C) * att_s.double().view(1, heads, C)).sum(-1)
    rd = (ref.view(n, heads, C) * att_d.double().view(1, heads, C)).sum(-1)
    assert_close(asrc, rs, rtol=1e-4, atol=1e-4)
    assert_close(adst, rd, rtol=1e-4, atol=1e-4)
    hb = rt.proj(xd, wd, out_dtype=torch.bfloat16)
    assert_close(hb, ref, rtol=1e-2, atol=1e-2)


@pytest.mark.parametrize(
    "n,k,f,heads,h_dtype",
    [
        (5000, 100, 256, 4, torch.bfloat16),
        (4099, 100, 47, 1, torch.bfloat16),
        (4099, 256, 47, 1, torch.float32),
        (1000, 64, 256, 2, torch.bfloat16),
        (1000, 64, 256, 16, torch.float32),
        (300, 128, 40, 1, torch.bfloat16),
        (100, 32, 64, 4, torch.bfloat16),
        (129, 96, 112, 7, torch.bfloat16),
    ],
)
def test_tensor_core_projection_epilogue(device, n, k, f, heads, h_dtype):
    """bf16 operands (the tcgen05 path): values, attention coefficients, and
    the output written only inside its [n, f] window of a wider row-padded
    buffer (the bulk-tensor stores clip rows and columns)."""
    from gnnc.b200 import runtime as rt

    g = torch.Generator().manual_seed(7 * n + f)
    x = torch.randn(n, k, generator=g).to(torch.bfloat16)
    w = (torch.randn(f, k, generator=g) / k**0.5).to(torch.bfloat16)
    att_s = torch.randn(f, generator=g)
    att_d = torch.randn(f, generator=g)
    xd = rt.empty_rows(n, k, torch.bfloat16, device)
    xd.copy_(x)
    wd = rt.empty_rows(f, k, torch.bfloat16, device)
    wd.copy_(w)
    sentinel = -1024.0
    # row stride: the 16-byte aligned width plus 24 spare columns
    big = torch.full((n + 3, (f + 7) // 8 * 8 + 24), sentinel, dtype=h_dtype, device=device)
    out = big[:n, :f]
    h, asrc, adst = rt.proj(xd, wd, att_src=att_s.to(device), att_dst=att_d.to(device),
                            heads=heads, out_dtype=h_dtype, out=out)
    assert h.data_ptr() == out.data_ptr()
    ref = x.double() @ w.double().t()
    tol = 1e-2 if h_dtype == torch.bfloat16 else 1e-4
    assert_close(out, ref, rtol=tol, atol=tol)
    C = f // heads
    rs = (ref.view(n, heads, C) * att_s.double().view(1, heads, C)).sum(-1)
    rd = (ref.view(n, heads, C) * att_d.double().view(1, heads, C)).sum(-1)
    assert_close(asrc, rs, rtol=1e-4, atol=1e-4)
    assert_close(adst, rd, rtol=1e-4, atol=1e-4)
    big = big.cpu()
    assert bool((big[:, f:] == sentinel).all()), "columns past f were written"
    assert bool((big[n:] == sentinel).all()), "rows past n were written"


def test_bounded_wait_gives_up_and_the_context_recovers(device):
    """The projection's bounded mbarrier wait, run on a barrier nothing arrives
    on with a 1 ms limit (gnnc_wait_selftest): gnnc_synchronize reports
    GNNC_ERR_TIMEOUT once, the report is cleared, and the next tensor-core
    projection on the same context succeeds and is correct."""
    import time

    from gnnc.b200 import runtime as rt
    from gnnc.b200._lib import ERR_TIMEOUT, GnncError

    ctx = rt.Context.get(device)
    t0 = time.monotonic()
    ctx.call("gnnc_wait_selftest", 1_000_000)
    with pytest.raises(GnncError) as exc:
        ctx.synchronize()
    assert exc.value.status == ERR_TIMEOUT and "bounded wait" in str(exc.value)
    assert time.monotonic() - t0 < 5.0
    ctx.synchronize()  # cleared
    g = torch.Generator().manual_seed(5)
    x = torch.randn(3000, 100, generator=g).to(torch.bfloat16)
    w = (torch.randn(256, 100, generator=g) * 0.1).to(torch.bfloat16)
    xd = rt.empty_rows(3000, 100, torch.bfloat16, device)
    xd.copy_(x)
    wd = rt.empty_rows(256, 100, torch.bfloat16, device)
    wd.copy_(w)
    h = rt.proj(xd, wd, out_dtype=torch.float32)
    ctx.synchronize()
    assert_close(h, x.double() @ w.double().t(), rtol=1e-4, atol=1e-4)
    with pytest.raises(ValueError):
        ctx.call("gnnc_wait_selftest", 0)
