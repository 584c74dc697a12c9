"""Test-only CPU oracle for the GCN / GAT aggregation path.

Importable only by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline
leg; the product path never calls it. See gnn_oracle.py for what is restated
and how it is pinned against the reference's known answers.
"""
