"""Device graph preparation vs the oracle: bit-exact CSR, degrees and weights."""

from __future__ import annotations

import numpy as np
import pytest
import torch
from conftest import GOLDEN
from gpu_util import random_graph

from oracle import gnn_oracle as O

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("self_loops", [True, False])
@pytest.mark.parametrize("dedupe", [True, False])
@pytest.mark.parametrize("n,e", [(1, 0), (5, 12), (300, 3000), (4096, 50000), (100003, 1_000_000)])
def test_csr_from_coo_bit_exact(device, n, e, self_loops, dedupe):
    from gnnc.b200 import runtime as rt

    ei = random_graph(n, e, seed=n + e, loops=3 if n > 1 else 0) if e else torch.zeros(2, 0, dtype=torch.long)
    rowptr, col, mult = rt.csr_from_coo(ei.to(device), n, self_loops=self_loops, dedupe=dedupe)
    r_rowptr, r_col, r_mult = O.csr_from_coo(ei.numpy(), n, self_loops=self_loops, dedupe=dedupe)
    assert np.array_equal(rowptr.cpu().numpy(), r_rowptr)
    assert np.array_equal(col.cpu().numpy(), r_col)
    if dedupe:
        assert np.array_equal(mult.cpu().numpy(), r_mult)


def test_csr_power_of_two_nodes_keep_last_loop(device):
    """N = 2^k: the (N-1, N-1) loop must not collide with the dropped-edge sentinel."""
    from gnnc.b200 import runtime as rt

    n = 1 << 12
    ei = torch.tensor([[n - 1, 0, n - 1, 5], [n - 1, n - 1, 0, 5]])
    rowptr, col, _ = rt.csr_from_coo(ei.to(device), n, self_loops=True, dedupe=True)
    r_rowptr, r_col, _ = O.csr_from_coo(ei.numpy(), n, self_loops=True, dedupe=True)
    assert np.array_equal(rowptr.cpu().numpy(), r_rowptr)
    assert np.array_equal(col.cpu().numpy(), r_col)


@pytest.mark.parametrize("g", range(4))
def test_gcn_norm_matches_torch_coalesce(device, g):
    """Device CSR + gcn_norm == torch coalesce of gcn_norm (fixture), bit for bit."""
    from gnnc.b200 import runtime as rt

    fx = np.load(GOLDEN / "csr_small.npz")
    n = int(fx[f"g{g}_n"])
    ei = torch.from_numpy(fx[f"g{g}_edge_index"]).to(device)
    rowptr, col, mult = rt.csr_from_coo(ei, n, self_loops=True, dedupe=True)
    _, _, w = rt.gcn_norm(rowptr, col, mult)
    assert np.array_equal(rowptr.cpu().numpy(), fx[f"g{g}_crow"])
    assert np.array_equal(col.cpu().numpy(), fx[f"g{g}_col"])
    assert np.array_equal(w.cpu().numpy().view(np.uint32), fx[f"g{g}_val"].view(np.uint32))


def test_gcn_norm_large_with_duplicates_bit_exact(device):
    from gnnc.b200 import runtime as rt

    n = 20000
    ei = random_graph(n, 200000, seed=11, heavy=((7, 30000),), dup_frac=0.3)
    rowptr, col, mult = rt.csr_from_coo(ei.to(device), n, self_loops=True, dedupe=True)
    deg, dinv, w = rt.gcn_norm(rowptr, col, mult)
    crow, rcol, val = O.normalized_csr_adj(ei, n)
    assert np.array_equal(rowptr.cpu().numpy(), crow.numpy())
    assert np.array_equal(col.cpu().numpy(), rcol.numpy())
    assert np.array_equal(w.cpu().numpy().view(np.uint32), val.numpy().view(np.uint32))
    rdeg, rdinv, _ = O.gcn_weights(crow.numpy(), rcol.numpy(), mult.cpu().numpy())
    assert np.array_equal(deg.cpu().numpy(), rdeg)
    assert np.array_equal(dinv.cpu().numpy().view(np.uint32), rdinv.view(np.uint32))


def test_device_normalized_csr_adj_matches_host(device):
    from gnnc.examples.util import normalized_csr_adj

    ei = random_graph(777, 5000, seed=2)
    host = normalized_csr_adj(ei, 777)
    dev = normalized_csr_adj(ei.to(device), 777)
    assert torch.equal(dev.crow_indices().cpu(), host.crow_indices())
    assert torch.equal(dev.col_indices().cpu(), host.col_indices())
    assert torch.equal(dev.values().cpu().view(torch.int32), host.values().view(torch.int32))


def test_out_of_range_endpoints_are_rejected(device):
    from gnnc.b200 import runtime as rt
    from gnnc.b200._lib import GnncInvalidArgument

    ei = torch.tensor([[0, 1, 9], [1, 2, 0]], device=device)
    with pytest.raises(GnncInvalidArgument):
        rt.csr_from_coo(ei, 5, self_loops=True, dedupe=True)
    ei = torch.tensor([[0, -1], [1, 2]], device=device)
    with pytest.raises(GnncInvalidArgument):
        rt.csr_from_coo(ei, 5, self_loops=False, dedupe=False)


def test_validate_catches_bad_columns_and_rowptr(device):
    from gnnc.b200 import runtime as rt
    from gnnc.b200._lib import GnncInvalidArgument

    rowptr = torch.tensor([0, 2, 3], dtype=torch.int32, device=device)
    col = torch.tensor([0, 1, 5], dtype=torch.int32, device=device)
    with pytest.raises(GnncInvalidArgument):
        rt.validate_csr(rowptr, col, 3)
    rt.validate_csr(rowptr, col, 6)
    bad = torch.tensor([0, 3, 2], dtype=torch.int32, device=device)
    with pytest.raises(GnncInvalidArgument):
        rt.validate_csr(bad, col, 6)
    with pytest.raises(GnncInvalidArgument):
        rt.Plan(bad)
