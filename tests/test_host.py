"""Host-side logic: phase pipeline, lowering, CLI exit codes, synthetic workloads."""

from __future__ import annotations

import os

import numpy as np
import pytest
import torch

from gnnc.compile import lower
from gnnc.examples import MODELS_DIR, available
from gnnc.ingress import get_model_and_data
from gnnc.pipeline.phase import PhaseNotReached, PhasePipeline


def test_available_models():
    assert available() == ["gat", "gcn", "sage"]


def test_phase_pipeline_stop_and_print():
    p = PhasePipeline()
    p.add_callable_phase("a", lambda m: m + 1, ("inc",))
    p.add_callable_phase("b", lambda m: m * 10, ("mul",))
    p.add_callable_phase("c", lambda m: m - 3)
    assert p.run(1)[0] == 17
    mod, trace = p.run(1, stop_after="b")
    assert mod == 20 and [t[0] for t in trace] == ["a", "b"]
    assert p.run(1, stop_before="b")[0] == 2
    seen = []
    p.run(1, print_ir_after=frozenset({"a"}), emit=seen.append)
    assert "IR after phase 'a'" in seen[0] and seen[0].endswith("2")
    seen.clear()
    p.run(1, print_ir_before=frozenset({"b"}), print_ir_after=frozenset({"c"}), emit=seen.append)
    assert len(seen) == 2 and seen[0].endswith("2") and seen[1].endswith("17")
    with pytest.raises(PhaseNotReached):
        p.run(1, stop_after="zz")
    with pytest.raises(PhaseNotReached):
        p.run(1, stop_before="b", print_ir_after=frozenset({"c"}))
    with pytest.raises(ValueError):
        p.run(1, stop_before="a", stop_after="b")
    with pytest.raises(ValueError):
        p.add_callable_phase("a", lambda m: m)
    q = PhasePipeline()
    q.add_callable_phase("d", lambda m: m)
    q.add_callable_phase("b", lambda m: m)
    with pytest.raises(ValueError):  # all or none: "d" is not taken either
        p.extend(q)
    assert p.names() == ["a", "b", "c"] and p.find("d") is None


@pytest.mark.parametrize("model_name", ["gcn", "gat", "sage"])
def test_lowering_fuses_epilogues(model_name):
    model, inputs = get_model_and_data(MODELS_DIR / f"{model_name}.py")
    prog, trace = lower(model, inputs, stop_after="b200-lower")
    assert [t[0] for t in trace] == ["import", "b200-lower"]
    assert [layer.kind for layer in prog.layers] == [model_name, model_name]
    first, last = prog.layers
    assert first.act == (2 if model_name == "gat" else 1)  # elu / relu
    assert last.log_softmax and not first.log_softmax
    if model_name == "gat":
        assert first.heads == 2 and first.concat and not last.concat
    if model_name == "sage":
        # lin_l with bias for the neighbour mean, lin_r for the root
        assert first.weight_root is not None and first.bias is not None
        assert tuple(first.weight.shape) == tuple(first.weight_root.shape) == (8, 4)


def test_lowering_rejects_unsupported_ops():
    from gnnc.nn import GCNConv

    class Odd(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.conv = GCNConv(4, 4, normalize=False)

        def forward(self, x, adj):
            return torch.tanh(self.conv(x, adj))

    with pytest.raises(NotImplementedError):
        lower(Odd(), (torch.randn(3, 4), None), stop_after="b200-lower")


def test_mlir_targets_are_import_errors():
    model, inputs = get_model_and_data(MODELS_DIR / "gcn.py")
    with pytest.raises(ImportError):
        lower(model, inputs, target="cpu")
    with pytest.raises(NotImplementedError):
        lower(model, inputs, target="tpu")


def test_bench_cli_exit_codes(capsys):
    from gnnc.tools.gnnc_bench import main

    assert main(["--model", "gcn", "--target", "cpu"]) == 3
    assert main(["--model", "gat", "--dataset", "c1"]) == 2  # c1 is a GCN workload
    assert main(["--model", "sage", "--dataset", "c2"]) == 2  # c2 is a GAT workload


def test_synthetic_c1_exact_shape_and_deterministic():
    from gnnc.examples import synthetic as S

    cfg = S.CONFIGS["c1"]
    ei = S.make_graph(cfg)
    assert ei.shape == (2, 10556)
    assert int((ei[0] == ei[1]).sum()) == 0
    keys = ei[0] * cfg.num_nodes + ei[1]
    assert torch.unique(keys).numel() == 10556
    # symmetric
    rev = ei[1] * cfg.num_nodes + ei[0]
    assert torch.equal(torch.sort(keys).values, torch.sort(rev).values)
    assert torch.equal(ei, S.make_graph(cfg))
    x = S.make_features(cfg)
    assert x.shape == (2708, 1433) and set(torch.unique(x).tolist()) <= {0.0, 1.0}
    assert abs(x.mean().item() - 0.0127) < 0.002


def test_synthetic_rmat_unique_count():
    from gnnc.examples import synthetic as S

    ei, m = S.rmat_unique_symmetric(1000, 5000, seed=3)
    assert m == 5000
    assert int((ei[0] == ei[1]).sum()) == 0
    assert ei.max() < 1000
    keys = ei[0] * 1000 + ei[1]
    assert torch.unique(keys).numel() == ei.size(1)


def test_config_model_power_law_tail():
    from gnnc.examples import synthetic as S

    ei = S.config_model_edges(20000, 100000, 2.1, seed=7)
    assert ei.size(1) == 200000
    deg = np.bincount(ei[1].numpy(), minlength=20000)
    assert deg.max() > 20 * deg.mean()  # heavy tail


def test_pinned_result_pool_never_hands_out_a_held_buffer(monkeypatch):
    """Result buffers are recycled only when the caller dropped every reference."""
    from gnnc.b200 import program

    made = []

    def fake_empty(shape, dtype, pin_memory):
        t = torch.zeros(shape, dtype=dtype)
        made.append(id(t))
        return t

    monkeypatch.setattr(program.torch, "empty", fake_empty)
    pool = program._PinnedResults()
    a = pool.take((4, 2), torch.float32)
    b = pool.take((4, 2), torch.float32)
    assert a is not b  # a is still held
    view = b[1:]
    del b
    c = pool.take((4, 2), torch.float32)
    assert c is not view._base  # a view keeps its buffer busy
    del a
    d = pool.take((4, 2), torch.float32)
    assert id(d) == made[0]  # a was dropped: recycled
    assert len(made) == 3


def test_graph_cache_key_survives_detach_and_tracks_updates():
    """run_jit hands the executable detached tensors; the graph cache must still
    hit for the same storage and miss after an in-place update."""
    from gnnc.b200.program import B200Executable

    ei = torch.randint(0, 10, (2, 30))
    k1 = B200Executable._graph_key(ei)
    assert B200Executable._graph_key(ei.detach()) == k1
    ei.add_(0)  # in-place: bumps the version counter
    assert B200Executable._graph_key(ei.detach()) != k1
    other = ei.clone()
    assert B200Executable._graph_key(other) != B200Executable._graph_key(ei)


def test_bench_roofline_uses_dram_bytes_of_the_current_kernel_only(tmp_path, monkeypatch):
    """bench.py's roofline: the primary figure is the ncu DRAM traffic of a
    capture whose recorded kernel-source hash matches the current source (one
    GPU only); otherwise the edge-gather model, labelled as an upper count."""
    import importlib
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, root)
    bench = importlib.import_module("bench")
    prof = tmp_path / "prof.txt"
    monkeypatch.setitem(bench.TRAFFIC_FILES, bench.WORKLOAD, prof)
    cur = bench.kernel_source_hash()
    prof.write_text(f"dram_bytes_per_launch_full_size: 20.0e9 bytes\nkernel_source_sha256_16: {cur}\n")
    r = bench.roofline("k", bench.WORKLOAD, 35.0e9, 4.0, 1)
    assert r["basis"] == "dram" and r["traffic"] == 20_000_000_000
    assert abs(r["achieved"] - 20.0e9 / 4e-3 / 1e9) < 1e-6 and r["frac"] == r["frac_dram"]
    assert r["algorithmic"]["achieved"] > r["achieved"]
    r2 = bench.roofline("k", bench.WORKLOAD, 17.5e9, 2.0, 2, 0.5)  # a rank's half of the edges
    assert r2["traffic"] == 10_000_000_000 and r2["basis"].startswith("dram (one-GPU capture")
    assert abs(r2["achieved"] - 10.0e9 / 2e-3 / 1e9) < 1e-6
    prof.write_text("dram_bytes_per_launch_full_size: 20.0e9 bytes\nkernel_source_sha256_16: 0000\n")
    r3 = bench.roofline("k", bench.WORKLOAD, 35.0e9, 4.0, 1)  # stale capture
    assert r3["traffic"] is None and not r3["traffic_source"]["current"]
