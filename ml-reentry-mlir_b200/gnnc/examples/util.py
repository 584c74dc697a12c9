"""COO -> normalised CSR adjacency, built the way the reference builds it.

normalized_csr_adj follows gnnc/examples/util.py:16-41 of the reference:
gcn_norm(edge_index, add_self_loops=True), flip to (row=dst, col=src),
sparse_coo_tensor(...).coalesce().to_sparse_csr(). PyG's gcn_norm is used when
torch_geometric is importable, else gnnc.nn.gcn_norm_edges (the same
arithmetic). Host tensors take this host path, like the reference; CUDA tensors
use the device kernels (gnnc_csr_from_coo + gnnc_gcn_norm), which produce the
same CSR bit for bit.
"""

from __future__ import annotations

import warnings

import torch


def _gcn_norm(edge_index: torch.Tensor, num_nodes: int):
    try:
        from torch_geometric.nn.conv.gcn_conv import gcn_norm
    except ImportError:
        from gnnc.nn import gcn_norm_edges

        return gcn_norm_edges(edge_index, num_nodes, add_self_loops=True)
    return gcn_norm(edge_index, num_nodes=num_nodes, add_self_loops=True)


def normalized_csr_adj(edge_index: torch.Tensor, num_nodes: int) -> torch.Tensor:
    """COO `edge_index` -> symmetric-normalised torch.sparse_csr_tensor (row = dst)."""
    if edge_index.is_cuda:
        from gnnc.b200 import runtime as rt

        rowptr, col, mult = rt.csr_from_coo(edge_index, num_nodes, self_loops=True, dedupe=True)
        _, _, w = rt.gcn_norm(rowptr, col, mult)
        with warnings.catch_warnings():
            warnings.filterwarnings("ignore", message=r".*Sparse CSR tensor support is in beta.*")
            return torch.sparse_csr_tensor(
                rowptr.to(torch.int64), col.to(torch.int64), w, (num_nodes, num_nodes),
                check_invariants=False,
            )
    ei, ew = _gcn_norm(edge_index, num_nodes)
    with warnings.catch_warnings(), torch.sparse.check_sparse_tensor_invariants(False):
        warnings.filterwarnings(
            "ignore", message=r".*Sparse CSR tensor support is in beta.*", category=UserWarning
        )
        coo = torch.sparse_coo_tensor(ei.flip(0), ew, (num_nodes, num_nodes))
        return coo.coalesce().to_sparse_csr()


def ring_edge_index(num_nodes: int) -> torch.Tensor:
    src = torch.arange(num_nodes)
    return torch.stack([src, (src + 1) % num_nodes])


def ring_csr_adj(num_nodes: int) -> torch.Tensor:
    """Small directed ring (every node degree >= 1) as a normalised CSR adjacency."""
    return normalized_csr_adj(ring_edge_index(num_nodes), num_nodes)
