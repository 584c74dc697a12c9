"""Reference GCN - GCNConv layers on a pre-normalised torch.sparse_csr adjacency.

Same model as the reference's gnnc/examples/models/gcn.py:32-51 (normalize=False,
add_self_loops=False; the symmetric normalisation is in the CSR values), with an
optional depth for the 3-layer workloads. KernelBench convention:
Model + get_init_inputs() + get_inputs().
"""

from __future__ import annotations

import torch
import torch.nn.functional as F
from torch import nn

from gnnc.examples.models._layers import GCNConv
from gnnc.examples.util import ring_csr_adj

_IN, _HIDDEN, _OUT, _NODES = 4, 8, 3, 5


class Model(nn.Module):
    def __init__(self, in_channels: int, hidden_channels: int, out_channels: int,
                 num_layers: int = 2) -> None:
        super().__init__()
        torch.manual_seed(0)
        dims = [in_channels] + [hidden_channels] * (num_layers - 1) + [out_channels]
        convs = [GCNConv(a, b, normalize=False, add_self_loops=False) for a, b in zip(dims, dims[1:])]
        # conv1, conv2 as in the reference; further layers conv3, ...
        for i, conv in enumerate(convs):
            setattr(self, f"conv{i + 1}", conv)
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
