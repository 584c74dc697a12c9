"""PyG-free dataset loaders (gnnc.datasets) on small files in the raw formats.

The real Cora / ogbn-arxiv files are not in this environment; these tests
write miniature files in the same layouts (Planetoid's pickled scipy matrices
and adjacency dict, OGB's gzipped CSVs) and check the tensors the loaders
rebuild against a direct construction of the same data.
"""

from __future__ import annotations

import gzip
import pickle

import numpy as np
import pytest
import scipy.sparse as sp
import torch


def _write_planetoid(root, name="cora"):
    raw = root / "planetoid" / name.capitalize() / "raw"
    raw.mkdir(parents=True)
    rng = np.random.default_rng(0)
    n_all, n_test, F, C = 6, 3, 5, 3
    allx = (rng.random((n_all, F)) < 0.4).astype(np.float32)
    tx = (rng.random((n_test, F)) < 0.4).astype(np.float32)
    ally = np.eye(C, dtype=np.float32)[rng.integers(0, C, n_all)]
    ty = np.eye(C, dtype=np.float32)[rng.integers(0, C, n_test)]
    test_index = np.array([8, 6, 7])  # unsorted, as in the real file
    graph = {0: [1, 2, 2], 1: [0, 1], 2: [0, 8], 6: [7], 7: [6, 3], 8: [2]}  # dup, self-loop
    objs = {"x": sp.csr_matrix(allx[:4]), "tx": sp.csr_matrix(tx), "allx": sp.csr_matrix(allx),
            "y": ally[:4], "ty": ty, "ally": ally, "graph": graph}
    for k, v in objs.items():
        with open(raw / f"ind.{name}.{k}", "wb") as f:
            pickle.dump(v, f)
    np.savetxt(raw / f"ind.{name}.test.index", test_index, fmt="%d")
    return allx, tx, ally, ty, test_index, graph


def test_planetoid_raw_files(tmp_path):
    from gnnc.datasets import load_cora

    allx, tx, ally, ty, test_index, graph = _write_planetoid(tmp_path)
    x, ei, y, nc = load_cora(tmp_path)
    xs = np.concatenate([allx, tx])
    ys = np.concatenate([ally, ty]).argmax(1)
    order = np.sort(test_index)
    xs[test_index] = xs[order].copy()
    ys[test_index] = ys[order].copy()
    assert np.array_equal(x.numpy(), xs) and np.array_equal(y.numpy(), ys)
    assert nc == 3 and x.dtype == torch.float32
    pairs = sorted({(a, b) for a, nb in graph.items() for b in nb if a != b})
    assert ei.tolist() == [[a for a, _ in pairs], [b for _, b in pairs]]


def _write_ogb(root, name, seed=1):
    raw = root / "ogb" / name / "raw"
    raw.mkdir(parents=True)
    rng = np.random.default_rng(seed)
    edges = rng.integers(0, 7, (11, 2))
    feat = rng.standard_normal((7, 4)).astype(np.float32)
    label = rng.integers(0, 5, (7, 1))
    for fname, arr, fmt in (("edge", edges, "%d"), ("node-feat", feat, "%.8e"),
                            ("node-label", label, "%d")):
        with gzip.open(raw / f"{fname}.csv.gz", "wt") as f:
            np.savetxt(f, arr, delimiter=",", fmt=fmt)
    return edges, feat, label


def test_ogb_raw_files(tmp_path):
    from gnnc.datasets import load_ogbn_arxiv

    edges, feat, label = _write_ogb(tmp_path, "ogbn_arxiv")
    x, ei, y, nc = load_ogbn_arxiv(tmp_path)
    assert np.array_equal(ei.numpy(), edges.T) and np.allclose(x.numpy(), feat)
    assert np.array_equal(y.numpy(), label.reshape(-1)) and nc == int(label.max()) + 1


def test_ogbn_products_adds_the_reverse_of_each_edge(tmp_path):
    """Stored edges are undirected: each (u, v) is followed by (v, u)."""
    from gnnc.datasets import load

    edges, feat, label = _write_ogb(tmp_path, "ogbn_products", seed=2)
    x, ei, y, nc = load("ogbn-products", tmp_path)
    want = []
    for u, v in edges.tolist():
        want += [(u, v), (v, u)]
    assert ei.t().tolist() == [list(p) for p in want]
    assert np.allclose(x.numpy(), feat) and np.array_equal(y.numpy(), label.reshape(-1))
    assert nc == int(label.max()) + 1


def test_missing_files_name_the_path(tmp_path):
    from gnnc.datasets import DatasetNotFound, load

    with pytest.raises(DatasetNotFound, match="ind.cora"):
        load("cora", tmp_path)
    with pytest.raises(ValueError):
        load("ogbn-arxiv", tmp_path)
    with pytest.raises(DatasetNotFound, match="ogbn_products"):
        load("ogbn-products", tmp_path)


def test_ingress_reads_the_raw_files(tmp_path, monkeypatch):
    """gnnc-bench --dataset cora without PyG: the loader's graph, normalised for GCN."""
    import gnnc.paths
    from gnnc.examples import MODELS_DIR
    from gnnc.ingress import get_model_and_data

    _write_planetoid(tmp_path)
    monkeypatch.setattr(gnnc.paths, "DATA_DIR", tmp_path)
    model, (x, adj) = get_model_and_data(MODELS_DIR / "gcn.py", "cora")
    assert adj.layout == torch.sparse_csr and adj.size(0) == x.size(0) == 9
    assert model.conv1.lin.weight.size(1) == x.size(1)


def test_ingress_reads_ogbn_products_for_gat(tmp_path, monkeypatch):
    """gnnc-bench --model gat --dataset ogbn-products: edge_index with both directions."""
    import gnnc.paths
    from gnnc.examples import MODELS_DIR
    from gnnc.ingress import get_model_and_data

    edges, feat, _ = _write_ogb(tmp_path, "ogbn_products", seed=3)
    monkeypatch.setattr(gnnc.paths, "DATA_DIR", tmp_path)
    model, (x, ei) = get_model_and_data(MODELS_DIR / "gat.py", "ogbn-products")
    assert ei.shape == (2, 2 * len(edges)) and x.shape == feat.shape
