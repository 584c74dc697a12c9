"""Pins the CPU oracle against the reference's known answers (no GPU)."""

from __future__ import annotations

import numpy as np
import pytest
import torch
from conftest import GOLDEN

from oracle import gnn_oracle as O


def test_gcn_toy_weights_replay_bit_exact():
    """Seeded init reproduces the GCN weights embedded in test/reference/gcn.raw.mlir."""
    from gnnc.examples.models import gcn

    fx = np.load(GOLDEN / "gcn_toy.npz")
    torch.manual_seed(0)
    m = gcn.Model(*gcn.get_init_inputs())
    assert np.array_equal(m.conv1.lin.weight.detach().numpy(), fx["w1"])
    assert np.array_equal(m.conv1.bias.detach().numpy(), fx["b1"])
    assert np.array_equal(m.conv2.lin.weight.detach().numpy(), fx["w2"])
    assert np.array_equal(m.conv2.bias.detach().numpy(), fx["b2"])


def test_gat_toy_weights_replay_bit_exact():
    """GATConv(4,2,heads=2) under seed 0 reproduces gat.1-raw-torch.mlir:137-139."""
    from gnnc.nn import GATConv

    fx = np.load(GOLDEN / "gat_toy.npz")
    torch.manual_seed(0)
    conv = GATConv(4, 2, heads=2, concat=True, add_self_loops=False, bias=False)
    assert np.array_equal(conv.lin.weight.detach().numpy(), fx["lin"])
    assert np.array_equal(conv.att_src.detach().numpy(), fx["att_src"])
    assert np.array_equal(conv.att_dst.detach().numpy(), fx["att_dst"])


def _dense_adj(crow, col, val, n):
    a = np.zeros((n, n))
    for r in range(n):
        for k in range(crow[r], crow[r + 1]):
            a[r, col[k]] += val[k]
    return a


def test_gcn_toy_oracle_matches_dense():
    """Layer order and bias placement of gcn.raw.mlir:4-21 on the ring fixture."""
    from gnnc.examples.models import gcn

    fx = np.load(GOLDEN / "gcn_toy.npz")
    csr = np.load(GOLDEN / "csr_small.npz")
    x, adj = gcn.get_inputs()
    crow, col, val = adj.crow_indices(), adj.col_indices(), adj.values()
    assert np.array_equal(crow.numpy(), csr["ring_crow"])
    assert np.array_equal(col.numpy(), csr["ring_col"])
    assert np.array_equal(val.numpy(), csr["ring_val"])
    torch.manual_seed(0)
    m = gcn.Model(*gcn.get_init_inputs())
    got = O.gcn_forward(m, x, crow, col, val).numpy()
    A = _dense_adj(crow.numpy(), col.numpy(), val.numpy(), 5)
    xd = x.double().numpy()
    h = np.maximum(A @ (xd @ fx["w1"].T.astype(np.float64)) + fx["b1"], 0)
    z = A @ (h @ fx["w2"].T.astype(np.float64)) + fx["b2"]
    ref = z - z.max(1, keepdims=True) - np.log(np.exp(z - z.max(1, keepdims=True)).sum(1, keepdims=True))
    np.testing.assert_allclose(got, ref, rtol=1e-5, atol=1e-6)


def test_gat_toy_oracle_matches_dense():
    """Op order of gat.1-raw-torch.mlir on its own 3-node graph and weights."""
    fx = np.load(GOLDEN / "gat_toy.npz")
    torch.manual_seed(0)
    from gnnc.nn import GATConv

    GATConv(4, 2, heads=2, concat=True, add_self_loops=False, bias=False)  # consume the init draws
    x = torch.randn(3, 4)  # experiments/gatconv/run.py:116
    ei = torch.from_numpy(fx["edge_index"])
    got = O.gat_layer(x, ei, torch.from_numpy(fx["lin"]), torch.from_numpy(fx["att_src"]),
                      torch.from_numpy(fx["att_dst"]), None, 2, 2, add_self_loops=False)
    # dense restatement in float64
    h = x.double().numpy() @ fx["lin"].T.astype(np.float64)
    h = h.reshape(3, 2, 2)
    a_s = (h * fx["att_src"].astype(np.float64)).sum(-1)
    a_d = (h * fx["att_dst"].astype(np.float64)).sum(-1)
    out = np.zeros((3, 2, 2))
    src, dst = fx["edge_index"]
    for d in range(3):
        ks = np.flatnonzero(dst == d)
        if ks.size == 0:
            continue
        e = a_s[src[ks]] + a_d[d]
        e = np.where(e > 0, e, 0.2 * e)
        p = np.exp(e - e.max(0))
        a = p / (p.sum(0) + 1e-16)
        out[d] = (a[:, :, None] * h[src[ks]]).sum(0)
    np.testing.assert_allclose(got.numpy(), out.reshape(3, 4), rtol=1e-5, atol=1e-6)


def test_softmax_spmm_known_answer():
    """experiments/gat-gpu-codegen/dumps/cpu.out.txt (printed to ~6 digits)."""
    crow, col, val, x = O.kat_softmax_inputs()
    y = np.load(GOLDEN / "kat_softmax.npz")["y"]
    got = O.softmax_aggregate(crow, col, val, torch.from_numpy(x), eps=0.0).numpy()
    np.testing.assert_allclose(got, y, rtol=1e-5, atol=5e-6)


def test_softmax_known_answer_needs_zero_drop():
    """The probe's dense->CSR convert drops the 29 zero-valued pattern entries;
    keeping them moves the answer far outside the printed precision."""
    i = np.arange(64)[:, None]
    j = np.arange(64)[None, :]
    val = (((i + 2 * j) % 13) - 6).astype(np.float32) * np.float32(0.3)
    mask = (i + j) % 11 == 0
    crow = np.concatenate([[0], np.cumsum(mask.sum(1))])
    rr, cc = np.nonzero(mask)
    _, _, _, x = O.kat_softmax_inputs()
    got = O.softmax_aggregate(crow, cc, val[rr, cc], torch.from_numpy(x)).numpy()
    y = np.load(GOLDEN / "kat_softmax.npz")["y"]
    assert np.abs(got - y).max() > 1e-2


@pytest.mark.parametrize("which", ["01", "05"])
def test_spmm_known_answers(which):
    crow, col, val, b = O.kat_spmm_inputs(which)
    y = np.load(GOLDEN / "kat_spmm.npz")[f"y{which}"]
    got = O.spmm_csr(crow, col, val, torch.from_numpy(b)).numpy()
    np.testing.assert_allclose(got, y, rtol=1e-6, atol=1e-5)


def test_ring_weights_are_torch_rounding():
    """Ring normalisation: fl(fl(1/sqrt(2))^2) = 0.49999997, not 0.5."""
    csr = np.load(GOLDEN / "csr_small.npz")
    assert np.all(csr["ring_val"] == np.float32(0.49999997))
    d = np.float32(1) / np.sqrt(np.float32(2))
    assert np.float32(d * d) == csr["ring_val"][0]


def test_dinv_formula_matches_torch_pow_bitwise():
    """deg.pow(-0.5) on CPU == IEEE 1/sqrt(deg) for every integer degree < 2^21."""
    deg = torch.arange(1, 1 << 21, dtype=torch.float32)
    a = deg.pow(-0.5).numpy()
    b = (np.float32(1) / np.sqrt(deg.numpy())).astype(np.float32)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


@pytest.mark.parametrize("g", range(4))
def test_numpy_csr_build_matches_torch_coalesce(g):
    """oracle.csr_from_coo + gcn_weights == torch coalesce of gcn_norm (bit-exact)."""
    csr = np.load(GOLDEN / "csr_small.npz")
    n = int(csr[f"g{g}_n"])
    rowptr, col, mult = O.csr_from_coo(csr[f"g{g}_edge_index"], n, self_loops=True, dedupe=True)
    _, _, w = O.gcn_weights(rowptr, col, mult)
    assert np.array_equal(rowptr, csr[f"g{g}_crow"])
    assert np.array_equal(col, csr[f"g{g}_col"])
    assert np.array_equal(w.view(np.uint32), csr[f"g{g}_val"].view(np.uint32))


def test_eager_layers_agree_with_oracle():
    """gnnc.nn eager GATConv / GCNConv == the oracle restatement."""
    from gnnc.nn import GATConv, GCNConv

    torch.manual_seed(3)
    n = 40
    ei = torch.randint(0, n, (2, 300))
    x = torch.randn(n, 12)
    conv = GATConv(12, 5, heads=3, concat=False)
    ref = O.gat_layer(x, ei, conv.lin.weight.detach(), conv.att_src.detach(), conv.att_dst.detach(),
                      conv.bias.detach(), 3, 5, concat=False)
    with torch.no_grad():
        torch.testing.assert_close(conv(x, ei), ref, rtol=1e-5, atol=1e-6)
    gconv = GCNConv(12, 6, normalize=False, add_self_loops=False)
    crow, col, val = O.normalized_csr_adj(ei, n)
    adj = torch.sparse_csr_tensor(crow, col, val, (n, n))
    with torch.no_grad():
        torch.testing.assert_close(
            gconv(x, adj),
            O.gcn_layer(x, crow, col, val, gconv.lin.weight.detach(), gconv.bias.detach()),
            rtol=1e-5, atol=1e-6,
        )


def test_rows_fp64_matches_layer():
    """The chunked float64 aggregation equals the op-by-op layer on a sample."""
    torch.manual_seed(5)
    n, H, C = 50, 2, 3
    ei = torch.randint(0, n, (2, 400))
    x = torch.randn(n, 7)
    W = torch.randn(H * C, 7)
    a_s, a_d = torch.randn(H, C), torch.randn(H, C)
    ref = O.gat_layer(x, ei, W, a_s, a_d, None, H, C)
    rowptr, col, _ = O.csr_from_coo(ei.numpy(), n, self_loops=True, dedupe=False)
    h = (x @ W.t()).view(n, H, C)
    asrc = (h * a_s).sum(-1)
    adst = (h * a_d).sum(-1)
    got = O.gat_rows_fp64(rowptr, col, h.view(n, -1), asrc, adst, H, chunk_edges=37)
    np.testing.assert_allclose(got.numpy(), ref.double().numpy(), rtol=1e-5, atol=1e-6)


def test_sage_toy_weights_replay_bit_exact():
    """The SAGE toy model under seed 0 reproduces the weights embedded in
    test/reference/sage.raw.mlir (PyG Linear's kaiming / uniform init, drawn
    twice per Linear as PyG does)."""
    from gnnc.examples.models import sage

    fx = np.load(GOLDEN / "sage_toy.npz")
    m = sage.Model(*sage.get_init_inputs())
    for i in (1, 2):
        conv = getattr(m, f"conv{i}")
        assert np.array_equal(conv.lin_l.weight.detach().numpy(), fx[f"wl{i}"])
        assert np.array_equal(conv.lin_l.bias.detach().numpy(), fx[f"bl{i}"])
        assert np.array_equal(conv.lin_r.weight.detach().numpy(), fx[f"wr{i}"])


def test_sage_toy_oracle_matches_dense_and_eager():
    """sage.raw.mlir:5-27 restated densely in float64: mean over the row's nonzero
    entries, lin_l with bias, plus lin_r, relu; layer 2; log_softmax."""
    from gnnc.examples.models import sage

    m = sage.Model(*sage.get_init_inputs())
    x, adj = sage.get_inputs()
    crow, col, val = adj.crow_indices(), adj.col_indices(), adj.values()
    n = x.size(0)
    a = torch.from_numpy(_dense_adj(crow.numpy(), col.numpy(), val.numpy(), n))
    nnz = (a != 0).sum(1).clamp_min(1).double()
    h = x.double()
    for i in (1, 2):
        conv = getattr(m, f"conv{i}")
        wl, bl = conv.lin_l.weight.double(), conv.lin_l.bias.double()
        wr = conv.lin_r.weight.double()
        h = ((a @ h) / nnz[:, None]) @ wl.t() + bl + h @ wr.t()
        h = torch.relu(h) if i == 1 else torch.log_softmax(h, dim=-1)
    ref = O.sage_forward(m, x, crow, col, val)
    np.testing.assert_allclose(ref.double().numpy(), h.detach().numpy(), rtol=1e-6, atol=1e-6)
    with torch.no_grad():
        eager = m(x, adj)
    np.testing.assert_allclose(eager.numpy(), ref.numpy(), rtol=1e-6, atol=1e-6)


def test_mean_weights_count_nonzero_values():
    crow = torch.tensor([0, 3, 3, 5])
    val = torch.tensor([0.5, 0.0, 2.0, 1.0, 3.0])
    w = O.mean_weights(crow, val)
    assert torch.equal(w, torch.tensor([0.25, 0.0, 1.0, 0.5, 1.5]))
    assert torch.equal(O.mean_weights(crow), torch.tensor([1 / 3, 1 / 3, 1 / 3, 0.5, 0.5]))
