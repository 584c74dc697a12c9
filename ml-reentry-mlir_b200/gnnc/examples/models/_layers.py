"""Layer classes for the example models: PyG's when installed, else gnnc.nn's."""

try:  # pragma: no cover - PyG is not installed in every environment
    from torch_geometric.nn import GATConv, GCNConv
except ImportError:
    from gnnc.nn import GATConv, GCNConv

__all__ = ["GATConv", "GCNConv"]
