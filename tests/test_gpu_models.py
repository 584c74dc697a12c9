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
    return O.gat_forward(model, x, graph)


@pytest.mark.parametrize("model_name", ["gcn", "gat"])
@pytest.mark.parametrize("dataset", [None, "c1", "c2"])
def test_compile_matches_oracle(device, model_name, dataset):
    if (model_name, dataset) in (("gcn", "c2"), ("gat", "c1")):
        pytest.skip("workload defined for the other model")
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
