"""Command-line tools (gnnc-bench)."""
