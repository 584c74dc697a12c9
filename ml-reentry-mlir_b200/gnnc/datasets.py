"""Dataset loaders that need neither torch_geometric nor ogb.

The reference loads Cora through PyG's Planetoid and ogbn-arxiv through OGB's
PygNodePropPredDataset (gnnc/ingress.py:52-83). Neither package is part of
this environment, so these functions read the same raw files those packages
download, from the same places under DATA_DIR, and rebuild the same tensors:

* Cora (Planetoid raw layout, DATA_DIR/planetoid/Cora/raw/ind.cora.*): the
  pickled x / tx / allx feature matrices and y / ty / ally one-hot labels, the
  adjacency dict `graph` and `test.index`. As PyG's read_planetoid_data does,
  the features are allx stacked on tx with the test rows put back in index
  order (x[test_index] = x[sorted(test_index)]); the edges are the dict's
  (node, neighbour) pairs with self-loops removed, then sorted and
  de-duplicated (coalesced): 2,708 nodes, 10,556 directed edges, 1,433
  binary features, 7 classes.
* ogbn-arxiv (OGB raw layout, DATA_DIR/ogb/ogbn_arxiv/raw/): edge.csv.gz
  (one "source,target" per line, kept directed as OGB does for this dataset),
  node-feat.csv.gz (128 floats per line) and node-label.csv.gz: 169,343 nodes,
  1,166,243 edges, 40 classes.
* ogbn-products (OGB raw layout, DATA_DIR/ogb/ogbn_products/raw/): the same
  three files; each undirected edge is stored once, and OGB's loader (its
  dataset table sets add_inverse_edge for this dataset) puts the reverse
  right after each stored edge: (u, v), (v, u), ... in file order. 2,449,029
  nodes, 61,859,140 directed edges, 100 features, 47 classes -- the graph whose
  shapes the synthetic c4 workload reproduces. The reference ships no loader
  for it (its dataset pre-download script leaves it for later).

Nothing is downloaded: a missing file raises DatasetNotFound (a ValueError,
so gnnc-bench exits with code 2) naming the path to put it at.
"""

from __future__ import annotations

import gzip
import pickle
from pathlib import Path

import numpy as np
import torch

__all__ = ["DatasetNotFound", "load", "load_cora", "load_ogbn_arxiv", "load_ogbn_products"]


class DatasetNotFound(ValueError):
    pass


def _need(path: Path) -> Path:
    if not path.exists():
        raise DatasetNotFound(f"dataset file not found: {path} (no download here: place the raw "
                              "files of the dataset at that path)")
    return path


def _unpickle(path: Path):
    with open(_need(path), "rb") as f:
        return pickle.load(f, encoding="latin1")


def _dense(m) -> np.ndarray:
    return np.asarray(m.todense() if hasattr(m, "todense") else m, dtype=np.float32)


def load_cora(root: Path, name: str = "cora"):
    """(x [N, F] float32, edge_index [2, E] int64, y [N] int64, num_classes)."""
    raw = Path(root) / "planetoid" / name.capitalize() / "raw"
    parts = {k: _unpickle(raw / f"ind.{name}.{k}") for k in ("x", "tx", "allx", "y", "ty", "ally",
                                                               "graph")}
    test_index = torch.from_numpy(
        np.loadtxt(_need(raw / f"ind.{name}.test.index"), dtype=np.int64).reshape(-1))
    sorted_test = test_index.sort().values
    tx, ty = _dense(parts["tx"]), np.asarray(parts["ty"], dtype=np.float32)
    if name == "citeseer":  # isolated test nodes: zero rows for the missing indices
        span = int(sorted_test[-1] - sorted_test[0]) + 1
        tx_ext = np.zeros((span, tx.shape[1]), dtype=np.float32)
        ty_ext = np.zeros((span, ty.shape[1]), dtype=np.float32)
        pos = (sorted_test - sorted_test[0]).numpy()
        tx_ext[pos], ty_ext[pos] = tx, ty
        tx, ty = tx_ext, ty_ext
    x = torch.from_numpy(np.concatenate([_dense(parts["allx"]), tx]))
    y = torch.from_numpy(np.concatenate([np.asarray(parts["ally"], dtype=np.float32), ty])).argmax(1)
    x[test_index] = x[sorted_test].clone()
    y[test_index] = y[sorted_test].clone()
    n = x.size(0)
    rows, cols = [], []
    for node, nbrs in parts["graph"].items():
        rows += [int(node)] * len(nbrs)
        cols += [int(v) for v in nbrs]
    src = torch.tensor(rows, dtype=torch.int64)
    dst = torch.tensor(cols, dtype=torch.int64)
    keep = src != dst
    key = torch.unique(src[keep] * n + dst[keep])  # coalesce: sorted by (src, dst), unique
    edge_index = torch.stack([key // n, key % n])
    return x, edge_index, y, int(y.max()) + 1


def _read_csv_gz(path: Path, dtype) -> np.ndarray:
    with gzip.open(_need(path), "rt") as f:
        return np.loadtxt(f, delimiter=",", dtype=dtype, ndmin=2)


def _load_ogb(root: Path, name: str, add_inverse: bool):
    raw = Path(root) / "ogb" / name / "raw"
    edges = _read_csv_gz(raw / "edge.csv.gz", np.int64)  # [E0, 2]
    x = torch.from_numpy(_read_csv_gz(raw / "node-feat.csv.gz", np.float32))
    y = torch.from_numpy(_read_csv_gz(raw / "node-label.csv.gz", np.int64)).reshape(-1)
    if add_inverse:  # (u, v) then (v, u) for every stored edge, in file order
        edges = np.stack([edges, edges[:, ::-1]], axis=1).reshape(-1, 2)
    edge_index = torch.from_numpy(np.ascontiguousarray(edges.T))
    return x, edge_index, y, int(y.max()) + 1


def load_ogbn_arxiv(root: Path):
    """(x [N, 128] float32, edge_index [2, E] int64, y [N] int64, num_classes)."""
    return _load_ogb(root, "ogbn_arxiv", add_inverse=False)


def load_ogbn_products(root: Path):
    """(x [N, 100] float32, edge_index [2, 2*E0] int64 with both directions of
    every stored edge, y [N] int64, num_classes)."""
    return _load_ogb(root, "ogbn_products", add_inverse=True)


def load(name: str, root: Path | None = None):
    """(x, edge_index, y, num_classes) of "cora", "ogbn-arxiv" or "ogbn-products"
    from DATA_DIR."""
    if root is None:
        from gnnc.paths import DATA_DIR

        root = DATA_DIR
    if name == "cora":
        return load_cora(root)
    if name == "ogbn-arxiv":
        return load_ogbn_arxiv(root)
    if name == "ogbn-products":
        return load_ogbn_products(root)
    raise ValueError(f"unknown dataset: {name}")
