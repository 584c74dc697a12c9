"""End-to-end drop-in: compile_executable(target="b200") + run_jit vs the oracle.

Mirrors the reference's test/integration/test_compile_matches_torch.py:21-56
(compile, run, compare), with the GAT cases it skips enabled, and the
synthetic workloads in place of the datasets."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import gnn_oracle as O

pytestmark = pytest.mark.gpu


def _run(model_name, dataset, dtype=None):
    from gnnc.compile import compile_executable
    from gnnc.examples import MODELS_DIR
    from gnnc.execution import run_jit
    from gnnc.ingress import get_model_and_data

    model, inputs = get_model_and_data(MODELS_DIR / f"{model_name}.py", dataset)
    model.eval()
    lowered, results = compile_executable(model, inputs, target="b200", dtype=dtype)
    (out,) = run_jit(lowered, results, inputs)
    assert out.device.type == "cpu" and tuple(out.shape) == results[0][0]
    return model, inputs, out


def assert_argmax_agrees(out: torch.Tensor, ref: torch.Tensor, tol: float) -> None:
    """Predictions agree exactly on every row whose oracle top-2 margin exceeds
    the numeric tolerance (closer pairs are ties within floating-point noise)."""
    top2 = ref.topk(2, dim=1).values
    decided = (top2[:, 0] - top2[:, 1]) > 2 * tol
    a, b = out.argmax(1), ref.argmax(1)
    bad = int((a[decided] != b[decided]).sum())
    assert bad == 0, f"{bad} decided rows disagree ({int((~decided).sum())} near-ties excluded)"


def _oracle(model_name, model, inputs):
    x, graph = inputs
    if model_name == "gcn":
        return O.gcn_forward(model, x, graph.crow_indices(), graph.col_indices(), graph.values())
    if model_name == "sage":
        return O.sage_forward(model, x, graph.crow_indices(), graph.col_indices(), graph.values())
    return O.gat_forward(model, x, graph)


@pytest.mark.parametrize("model_name", ["gcn", "gat", "sage"])
@pytest.mark.parametrize("dataset", [None, "c1", "c2"])
def test_compile_matches_oracle(device, model_name, dataset):
    if (model_name, dataset) in (("gcn", "c2"), ("gat", "c1"), ("sage", "c2")):
        pytest.skip("workload defined for another model")
    model, inputs, out = _run(model_name, dataset)
    ref = _oracle(model_name, model, inputs)
    np.testing.assert_allclose(out.numpy(), ref.numpy(), rtol=1e-4, atol=1e-4)
    assert_argmax_agrees(out, ref, 1e-4)


def test_compile_matches_eager_model(device):
    """The reference's own check: compiled output vs the model's eager forward."""
    model, inputs, out = _run("gat", "c2")
    with torch.no_grad():
        ref = model(*inputs)
    np.testing.assert_allclose(out.numpy(), ref.numpy(), rtol=1e-3, atol=1e-4)


@pytest.mark.parametrize("dataset,dtype,tol", [("c3", None, 1e-4), ("c3-bf16", None, 2e-2)])
def test_c3_rmat_three_layer_gat(device, dataset, dtype, tol):
    model, inputs, out = _run("gat", dataset, dtype)
    x, ei = inputs
    ref = O.gat_forward(model, x.to(torch.float32), ei)
    np.testing.assert_allclose(out.numpy(), ref.numpy(), rtol=tol, atol=tol)
    assert_argmax_agrees(out, ref, tol)


@pytest.mark.parametrize("model_name,dataset", [("gat", "c3-bf16"), ("gcn", "c1")])
def test_host_result_copied_in_row_chunks(device, model_name, dataset):
    """With host inputs the last aggregation runs in edge-balanced row ranges,
    each copied to the host as soon as it is done; every row takes the same
    kernel path as in the single launch, so the result is bit-identical to the
    device-resident forward."""
    from gnnc.compile import compile_executable
    from gnnc.examples import MODELS_DIR
    from gnnc.execution import run_jit
    from gnnc.ingress import get_model_and_data

    model, inputs = get_model_and_data(MODELS_DIR / f"{model_name}.py", dataset)
    model.eval()
    lowered, results = compile_executable(model, inputs, target="b200")
    lowered.host_chunk_min_edges = 64
    (out,) = run_jit(lowered, results, inputs)
    x, graph = inputs
    g = lowered._graph_for(graph.to(device) if graph.layout == torch.strided else graph,
                           x.size(0), lowered.program.layers[-1])
    assert len(g.row_chunks(lowered.host_chunks)) > 1
    dev = lowered.run_device(x.to(device), graph.to(device) if graph.layout == torch.strided
                             else graph).cpu()
    assert torch.equal(out, dev)


@pytest.mark.parametrize("model_name,dataset,chunk_edges", [("gat", "c3-bf16", 64),
                                                            ("gcn", "c1", 1 << 21)])
def test_batch_stream_matches_one_call_at_a_time(device, model_name, dataset, chunk_edges):
    """run_stream over four host batches (page-locked and pageable, all
    different) yields, batch for batch, exactly what one call at a time
    returns, with the results of the earlier batches held by the caller while
    the later ones run (so every result buffer stays its own)."""
    from gnnc.compile import compile_executable
    from gnnc.examples import MODELS_DIR
    from gnnc.execution import run_jit
    from gnnc.ingress import get_model_and_data

    model, inputs = get_model_and_data(MODELS_DIR / f"{model_name}.py", dataset)
    model.eval()
    lowered, results = compile_executable(model, inputs, target="b200")
    lowered.host_chunk_min_edges = chunk_edges
    x, graph = inputs
    gen = torch.Generator().manual_seed(5)
    xs = [x, torch.randn(x.shape, generator=gen).to(x.dtype).pin_memory(),
          (x.float() * -0.5).to(x.dtype), torch.randn(x.shape, generator=gen).to(x.dtype)]
    streamed = list(lowered.run_stream(iter(xs), graph))
    assert len(streamed) == len(xs)
    for k, xb in enumerate(xs):
        (one,) = run_jit(lowered, results, (xb, graph))
        assert streamed[k].device.type == "cpu"
        assert torch.equal(streamed[k], one), f"batch {k}"
    assert not torch.equal(streamed[0], streamed[1])
    assert list(lowered.run_stream(iter([]), graph)) == []


def test_sage_on_edge_index_matches_eager(device):
    """SAGEConv fed an edge_index (PyG's other input form): the mean runs over
    incoming edges, duplicates counted, no self-loops added."""
    from gnnc.compile import compile_executable
    from gnnc.examples.models import sage
    from gnnc.examples.synthetic import CONFIGS, make_features, make_graph
    from gnnc.execution import run_jit

    cfg = CONFIGS["c1"]
    ei = make_graph(cfg)
    ei = torch.cat([ei, ei[:, :500]], dim=1)  # duplicates
    x = make_features(cfg)
    model = sage.Model(cfg.in_channels, 32, cfg.out_channels).eval()
    lowered, results = compile_executable(model, (x, ei), target="b200")
    (out,) = run_jit(lowered, results, (x, ei))
    with torch.no_grad():
        ref = model(x, ei)
    np.testing.assert_allclose(out.numpy(), ref.numpy(), rtol=1e-4, atol=1e-4)
    assert_argmax_agrees(out, ref, 1e-4)


def test_sage_power_law_bf16_rows_match_oracle(device):
    """A 3-layer SAGE on a 60k-node power-law graph with bf16 features
    (256-wide rows: the specialised edge loop plus the root term; a 47-wide last
    layer: the narrow loop) against the oracle."""
    from gnnc.compile import compile_executable
    from gnnc.examples.models import sage
    from gnnc.examples.synthetic import config_model_edges
    from gnnc.examples.util import normalized_csr_adj
    from gnnc.execution import run_jit

    n = 60_000
    ei = config_model_edges(n, 400_000, 2.1, seed=3)
    adj = normalized_csr_adj(ei, n)
    g = torch.Generator().manual_seed(4)
    x = torch.randn(n, 100, generator=g).to(torch.bfloat16)
    model = sage.Model(100, 256, 47, num_layers=3).eval()
    lowered, results = compile_executable(model, (x, adj), target="b200")
    (out,) = run_jit(lowered, results, (x, adj))
    ref = O.sage_forward(model, x.to(torch.float32), adj.crow_indices(), adj.col_indices(),
                         adj.values())
    np.testing.assert_allclose(out.numpy(), ref.numpy(), rtol=2e-2, atol=2e-2)


@pytest.mark.parametrize("model_name,dataset", [("gcn", "c1"), ("gat", "c2"), ("gat", "c3-bf16"),
                                                ("sage", "c1")])
def test_cuda_graph_replay_matches_eager(device, model_name, dataset):
    """Small graphs replay a captured CUDA graph of the forward: the result is
    bit-identical to the eager forward, and a new input reaches the graph."""
    from gnnc.compile import compile_executable
    from gnnc.examples import MODELS_DIR
    from gnnc.execution import run_jit
    from gnnc.ingress import get_model_and_data

    model, inputs = get_model_and_data(MODELS_DIR / f"{model_name}.py", dataset)
    model.eval()
    lowered, results = compile_executable(model, inputs, target="b200")
    x, graph = inputs
    for scale in (1.0, 0.5):
        xs = (x.float() * scale).to(x.dtype)
        (out,) = run_jit(lowered, results, (xs, graph))
        assert lowered.cuda_graph_error is None and len(lowered._cuda_graphs) == 1
        eager = lowered.run_device(xs.to(device), graph.to(device) if graph.layout == torch.strided
                                   else graph)
        assert torch.equal(out, eager.cpu())
