"""GraphSAGE: SAGEConv layers on the normalised CSR adjacency.

Follows the reference's SAGE model (gnnc/examples/models/sage.py): SAGEConv
(mean aggregation, root weight) -> ReLU -> SAGEConv -> log_softmax, fed the
same normalised CSR adjacency as the GCN model. Its toy inputs are the ring
graph of 5 nodes and x = randn(5, 4) after torch.manual_seed(0); the seeded
weights are the ones embedded in test/reference/sage.raw.mlir.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F
from torch import nn

from gnnc.examples.models._layers import SAGEConv
from gnnc.examples.util import ring_csr_adj

_IN, _HIDDEN, _OUT, _NODES = 4, 8, 3, 5


class Model(nn.Module):
    def __init__(self, in_channels: int, hidden_channels: int, out_channels: int,
                 num_layers: int = 2) -> None:
        super().__init__()
        torch.manual_seed(0)
        dims = [in_channels] + [hidden_channels] * (num_layers - 1) + [out_channels]
        # conv1, conv2 as in the reference; further layers conv3, ...
        for i, (a, b) in enumerate(zip(dims, dims[1:])):
            setattr(self, f"conv{i + 1}", SAGEConv(a, b))
        self.num_layers = num_layers

    def forward(self, x: torch.Tensor, adj: torch.Tensor) -> torch.Tensor:
        for i in range(1, self.num_layers):
            x = F.relu(getattr(self, f"conv{i}")(x, adj))
        return F.log_softmax(getattr(self, f"conv{self.num_layers}")(x, adj), dim=-1)


def get_init_inputs():
    return (_IN, _HIDDEN, _OUT)


def get_inputs():
    torch.manual_seed(0)
    x = torch.randn(_NODES, _IN)
    return (x, ring_csr_adj(_NODES))
