"""Reference GAT - GATConv layers on an edge_index (PyG convention).

The reference has no gat.py (its GAT cases are skipped, test/integration/
test_compile_matches_torch.py:10,33-35); this model follows the GAT it times in
experiments/pyg-baseline/run.py:78-88: GATConv(heads, concat=True) -> ELU ->
... -> GATConv(1 head, concat=False) -> log_softmax. GATConv adds self-loops
itself (add_self_loops=True). KernelBench convention.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F
from torch import nn

from gnnc.examples.models._layers import GATConv
from gnnc.examples.util import ring_edge_index

_IN, _HIDDEN, _OUT, _NODES, _HEADS = 4, 8, 3, 5, 2


class Model(nn.Module):
    def __init__(self, in_channels: int, hidden_channels: int, out_channels: int,
                 heads: int = _HEADS, num_layers: int = 2) -> None:
        super().__init__()
        torch.manual_seed(0)
        dim = in_channels
        for i in range(1, num_layers):
            setattr(self, f"conv{i}", GATConv(dim, hidden_channels, heads=heads, concat=True))
            dim = hidden_channels * heads
        setattr(self, f"conv{num_layers}", GATConv(dim, out_channels, heads=1, concat=False))
        self.num_layers = num_layers

    def forward(self, x: torch.Tensor, edge_index: torch.Tensor) -> torch.Tensor:
        for i in range(1, self.num_layers):
            x = F.elu(getattr(self, f"conv{i}")(x, edge_index))
        return F.log_softmax(getattr(self, f"conv{self.num_layers}")(x, edge_index), dim=-1)


def get_init_inputs():
    return (_IN, _HIDDEN, _OUT)


def get_inputs():
    torch.manual_seed(0)
    x = torch.randn(_NODES, _IN)
    return (x, ring_edge_index(_NODES))
