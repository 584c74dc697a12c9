"""The row-sampled parity checker (oracle/parity.py) agrees with the
whole-graph oracle layers on small graphs (CPU only)."""

from __future__ import annotations

import numpy as np
import torch
from gpu_util import random_graph

from oracle import gnn_oracle as O
from oracle import parity as P


def _csr(ei, n):
    rowptr, col, _ = O.csr_from_coo(ei.numpy(), n, self_loops=True, dedupe=False)
    return torch.from_numpy(rowptr), torch.from_numpy(col)


def test_sample_rows_takes_every_hub_and_is_seeded():
    n = 400
    ei = random_graph(n, 3000, 1, heavy=((7, 300), (11, 120)))
    rowptr, _ = _csr(ei, n)
    a = P.sample_rows(rowptr, sample=50, hub_degree=100, seed=3, extra=(5,))
    b = P.sample_rows(rowptr, sample=50, hub_degree=100, seed=3, extra=(5,))
    assert torch.equal(a, b) and bool((a.diff() > 0).all())
    assert {7, 11, 5} <= set(a.tolist()) and 52 <= a.numel() <= 53


def test_gat_rows_match_whole_graph_layer():
    n, H, C = 300, 4, 8
    ei = random_graph(n, 2500, 2, heavy=((3, 400),))
    g = torch.Generator().manual_seed(2)
    x = torch.randn(n, 20, generator=g, dtype=torch.float64)
    W = torch.randn(H * C, 20, generator=g, dtype=torch.float64) * 0.3
    a_s = torch.randn(1, H, C, generator=g, dtype=torch.float64) * 0.3
    a_d = torch.randn(1, H, C, generator=g, dtype=torch.float64) * 0.3
    bias = torch.randn(H * C, generator=g, dtype=torch.float64)
    full = O.gat_layer(x, ei, W, a_s, a_d, bias, H, C, act="elu")
    rowptr, col = _csr(ei, n)
    rows = P.sample_rows(rowptr, sample=60, hub_degree=50, seed=0)
    got = P.gat_conv_rows_fp64(x, rowptr, col, rows, W, a_s, a_d, bias, H, act="elu")
    np.testing.assert_allclose(got.numpy(), full[rows].numpy(), rtol=1e-12, atol=1e-12)
    last = O.gat_layer(x, ei, W[:C], a_s[:, :1], a_d[:, :1], bias[:C], 1, C, concat=False,
                       log_softmax=True)
    got = P.gat_conv_rows_fp64(x, rowptr, col, rows, W[:C], a_s[:, :1], a_d[:, :1], bias[:C], 1,
                               concat=False, log_softmax=True)
    np.testing.assert_allclose(got.numpy(), last[rows].numpy(), rtol=1e-12, atol=1e-12)


def test_gcn_rows_match_whole_graph_layer():
    n = 300
    ei = random_graph(n, 2500, 4, heavy=((9, 200),))
    crow, col, val = O.normalized_csr_adj(ei, n)
    g = torch.Generator().manual_seed(4)
    x = torch.randn(n, 16, generator=g, dtype=torch.float64)
    W = torch.randn(10, 16, generator=g, dtype=torch.float64)
    bias = torch.randn(10, generator=g, dtype=torch.float64)
    full = O.gcn_layer(x, crow, col, val.double(), W, bias, act="relu")
    rows = P.sample_rows(crow, sample=40, hub_degree=60, seed=1)
    got = P.gcn_conv_rows_fp64(x, crow, col, val, rows, W, bias, act="relu")
    np.testing.assert_allclose(got.numpy(), full[rows].numpy(), rtol=1e-12, atol=1e-12)


def test_compare_and_argmax_verdicts():
    ref = torch.tensor([[1.0, 0.5, -2.0], [0.30, 0.29, 0.0]], dtype=torch.float64)
    got = ref.clone()
    got[1, 0], got[1, 1] = 0.29, 0.30  # a flip inside a near-tie
    c = P.compare(got, ref, rtol=2e-2, atol=2e-2)
    assert c["pass"] and abs(c["max_abs_err"] - 0.01) < 1e-12
    a = P.argmax_agreement(got, ref, c["max_abs_err"])
    assert a["pass"] and a["near_ties"] == 1 and a["disagree"] == 1
    assert abs(a["max_margin_of_disagreeing_rows"] - 0.01) < 1e-12
    got[0, 1] = 1.2  # a decided row flips
    assert not P.compare(got, ref, rtol=2e-2, atol=2e-2)["pass"]
    assert not P.argmax_agreement(got, ref, 0.01)["pass"]
