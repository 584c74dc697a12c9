"""gnnc - GNN compiler front end with a B200 (sm_100a) backend.

Mirrors the entry points of the reference GNNC package for the GCN / GAT
aggregation path: gnnc.compile.compile_executable / lower, gnnc.execution.run_jit,
and the gnnc-bench CLI (gnnc.tools.gnnc_bench). The `b200` target runs
hand-written CUDA kernels from libgnnc_b200.so; see gnnc.b200.
"""

from __future__ import annotations

__version__ = "0.1.0"


def get_context():
    """The reference returns its memoised MLIR context here (gnnc/__init__.py:23-39).

    The B200 target needs no MLIR context; phases receive None."""
    return None
