"""Peer memory through the C ABI: gnnc_peer_export / gnnc_peer_open / gnnc_peer_close.

A second process maps the first process's input block (CUDA IPC; both on
cuda:0, so the test needs one GPU) and runs the projection with its x operand
read through the mapping; the result must equal the projection of the same
rows read locally, bit for bit (same kernel, same operands), and rows gathered
from the mapping (gnnc_gather_rows) equal the same rows of the block. These
are the read paths the multi-GPU layer uses for remote input rows."""

from __future__ import annotations

import os
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _weights(K, F, H, dtype):
    g = torch.Generator().manual_seed(5)
    W = torch.randn(F, K, generator=g).to(dtype)
    a_s = torch.randn(F, generator=g) * 0.1
    a_d = torch.randn(F, generator=g) * 0.1
    return W, a_s, a_d


def _child(handle, offset, rows, cols, ld, dtype_name, out_path):
    sys.path[:0] = [ROOT, os.path.join(ROOT, "ml-reentry-mlir_b200")]
    import torch

    from gnnc.b200 import runtime as rt

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    dtype = getattr(torch, dtype_name)
    ptr = rt.peer_open(dev, handle, offset)
    xv = rt.DeviceRows(ptr, rows, cols, ld, dtype, dev)
    W, a_s, a_d = _weights(cols, 256, 4, dtype)
    h, asrc, adst = rt.proj(xv, W.to(dev), att_src=a_s.to(dev), att_dst=a_d.to(dev), heads=4,
                            out_dtype=torch.bfloat16)
    # a row slice of the mapping reads the right rows
    h2 = rt.proj(xv[rows // 3 : rows // 3 + 100], W.to(dev), out_dtype=torch.bfloat16)
    # whole padded rows gathered straight from the mapping (plain loads)
    idx = torch.randint(0, rows, (999,), generator=torch.Generator().manual_seed(9),
                        dtype=torch.int32).to(dev)
    g = rt.gather_rows(xv, idx, torch.zeros((999, ld), dtype=dtype, device=dev))
    rt.Context.get(dev).synchronize()
    torch.save({"h": h.cpu(), "asrc": asrc.cpu(), "adst": adst.cpu(), "h2": h2.cpu(),
                "g": g.cpu(), "idx": idx.cpu()}, out_path)
    rt.peer_close(dev, ptr, offset)


@pytest.mark.timeout(300)
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_projection_reads_a_peer_mapped_buffer(device, tmp_path, dtype):
    import torch.multiprocessing as mp

    from gnnc.b200 import runtime as rt

    rows, cols = 5000, 100
    ld = rt.row_stride(cols, dtype)
    g = torch.Generator().manual_seed(3)
    block = torch.zeros((rows + 17, ld), dtype=dtype)
    block[:rows, :cols] = torch.randn(rows, cols, generator=g).to(dtype)
    x = block.to(device)
    handle, offset = rt.peer_export(x)
    assert len(handle) == rt.PEER_HANDLE_BYTES
    out_path = str(tmp_path / "child.pt")
    ctx = mp.get_context("spawn")
    p = ctx.Process(target=_child, args=(handle, offset, rows, cols, ld,
                                         str(dtype).split(".")[1], out_path))
    p.start()
    p.join(240)
    assert p.exitcode == 0, f"child exited with {p.exitcode}"
    got = torch.load(out_path)
    W, a_s, a_d = _weights(cols, 256, 4, dtype)
    xl = x[:rows, :cols]
    h, asrc, adst = rt.proj(xl, W.to(device), att_src=a_s.to(device), att_dst=a_d.to(device),
                            heads=4, out_dtype=torch.bfloat16)
    h2 = rt.proj(xl[rows // 3 : rows // 3 + 100], W.to(device), out_dtype=torch.bfloat16)
    assert torch.equal(got["h"], h.cpu())
    assert torch.equal(got["asrc"], asrc.cpu())
    assert torch.equal(got["adst"], adst.cpu())
    assert torch.equal(got["h2"], h2.cpu())
    bits = torch.int16 if dtype == torch.bfloat16 else torch.int32
    assert torch.equal(got["g"].view(bits), block.view(bits)[got["idx"].long()])


def test_peer_export_rejects_host_memory(device):
    import ctypes

    from gnnc.b200 import _lib
    from gnnc.b200 import runtime as rt

    ctx = rt.Context.get(device)
    host = ctypes.create_string_buffer(4096)
    handle = ctypes.create_string_buffer(rt.PEER_HANDLE_BYTES)
    off = ctypes.c_uint64()
    st = ctx.lib.gnnc_peer_export(ctx.handle, ctypes.addressof(host), handle, ctypes.byref(off))
    assert st == _lib.ERR_INVALID
    with pytest.raises(ValueError):
        rt.peer_export(torch.zeros(4))


def test_gather_rows_packs_whole_rows(device):
    """gnnc_gather_rows: dst[i] = src[idx[i]], padded rows copied whole; an
    index past the table is skipped and reported by the next synchronize."""
    from gnnc.b200 import runtime as rt
    from gnnc.b200._lib import GnncInvalidArgument

    src = rt.empty_rows(1000, 100, torch.bfloat16, device)
    src.copy_(torch.randn(1000, 100, device=device))
    base = src.as_strided((1000, src.stride(0)), (src.stride(0), 1))
    idx = torch.randint(0, 1000, (777,), device=device, dtype=torch.int32)
    out = torch.zeros((777, src.stride(0)), dtype=torch.bfloat16, device=device)
    rt.gather_rows(base, idx, out)
    # the padding columns hold whatever the allocation held (NaN bit patterns
    # among them): compare the rows as bits
    bits = base.view(torch.int16)
    assert torch.equal(out.view(torch.int16), bits[idx.long()])
    bad = torch.tensor([3, 5000, 7], device=device, dtype=torch.int32)
    out2 = torch.zeros((3, src.stride(0)), dtype=torch.bfloat16, device=device)
    rt.gather_rows(base, bad, out2)
    with pytest.raises(GnncInvalidArgument):
        rt.Context.get(device).synchronize()
    got = out2.view(torch.int16)
    assert torch.equal(got[0], bits[3]) and torch.equal(got[2], bits[7])
    assert bool((got[1] == 0).all())
