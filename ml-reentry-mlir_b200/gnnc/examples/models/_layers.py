"""Layer classes for the example models: PyG's when installed, else gnnc.nn's."""

try:  # pragma: no cover - PyG is not installed in every environment
    from torch_geometric.nn import GATConv, GCNConv, SAGEConv
except ImportError:
    from gnnc.nn import GATConv, GCNConv, SAGEConv

__all__ = ["GATConv", "GCNConv", "SAGEConv"]
