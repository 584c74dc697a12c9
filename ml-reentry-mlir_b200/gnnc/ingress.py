"""From user-land Python to a (model, forward_inputs) pair.

`get_model_and_data(model_file, dataset)` keeps the reference's behaviour
(gnnc/ingress.py:25-49): load the model file, take inputs from its own
get_inputs()/get_init_inputs() or from a named dataset, seed 0, build the model.
Named datasets are the reference's real ones ("cora", "ogbn-arxiv", loaded
through PyG/OGB when installed), "ogbn-products" (the real graph behind the c4
shapes) and the seeded synthetic workloads of gnnc.examples.synthetic
("c1" ... "c5"). The torch-mlir import
(import_as_raw_ir) belongs to the MLIR targets and is not part of this build.
"""

from __future__ import annotations

import importlib.util
from pathlib import Path

import torch

_DEFAULT_HIDDEN = 64


def _load_module(model_file: Path):
    spec = importlib.util.spec_from_file_location("_gnnc_model", str(model_file))
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    return module


def get_model_and_data(model_file: Path, dataset: str | None = None):
    module = _load_module(Path(model_file))
    if dataset is None:
        forward_inputs = module.get_inputs()
        init_inputs = module.get_init_inputs()
        init_kwargs = {}
    else:
        forward_inputs, init_inputs, init_kwargs = _dataset_inputs(Path(model_file).stem, dataset)
    torch.manual_seed(0)
    return module.Model(*init_inputs, **init_kwargs), forward_inputs


def synthetic_inputs(model_name: str, name: str):
    """(forward_inputs, init_inputs, init_kwargs) of a synthetic workload."""
    from gnnc.examples import synthetic as S
    from gnnc.examples.util import normalized_csr_adj

    # GraphSAGE runs on the GCN workloads' graphs and features (the reference
    # feeds its SAGE model the GCN model's normalised CSR adjacency).
    graph_model = "gcn" if model_name == "sage" else model_name
    key = name
    if name == "c4":
        key = f"c4-{graph_model}"
    if key not in S.CONFIGS:
        raise ValueError(f"unknown dataset: {name}")
    cfg = S.CONFIGS[key]
    if cfg.model != graph_model:
        raise ValueError(f"workload {name} is defined for model {cfg.model!r}, not {model_name!r}")
    ei = S.make_graph(cfg)
    x = S.make_features(cfg)
    if graph_model == "gcn":
        graph = normalized_csr_adj(ei, cfg.num_nodes)
        return (x, graph), (cfg.in_channels, cfg.hidden, cfg.out_channels), {"num_layers": cfg.num_layers}
    kw = {"heads": cfg.heads, "num_layers": cfg.num_layers}
    return (x, ei), (cfg.in_channels, cfg.hidden, cfg.out_channels), kw


def _dataset_inputs(model_name: str, dataset: str):
    from gnnc.examples.util import normalized_csr_adj
    from gnnc.paths import DATA_DIR

    if dataset not in ("cora", "ogbn-arxiv", "ogbn-products"):
        return synthetic_inputs(model_name, dataset)
    try:  # the reference's loaders, when PyG / OGB are installed
        if dataset == "cora":
            from torch_geometric.datasets import Planetoid

            ds = Planetoid(root=str(DATA_DIR / "planetoid"), name="Cora")
        else:
            from ogb.nodeproppred import PygNodePropPredDataset

            ds = PygNodePropPredDataset(name=dataset, root=str(DATA_DIR / "ogb"))
    except ImportError:  # the same raw files, read without them
        from gnnc.datasets import load

        x, edge_index, _, num_classes = load(dataset, DATA_DIR)
        graph = (normalized_csr_adj(edge_index, x.size(0)) if model_name in ("gcn", "sage")
                 else edge_index)
        return (x, graph), (x.size(1), _DEFAULT_HIDDEN, num_classes), {}
    data = ds[0]
    graph = (normalized_csr_adj(data.edge_index, data.num_nodes) if model_name in ("gcn", "sage")
             else data.edge_index)
    return (data.x, graph), (ds.num_node_features, _DEFAULT_HIDDEN, ds.num_classes), {}
