"""B200 backend: C-ABI bindings (_lib), device ops (runtime), kernel programs (program)."""
