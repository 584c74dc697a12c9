"""execution - run a compiled module (same entry point as gnnc/execution/__init__.py:25-69).

`run_jit(lowered, results, inputs)` invokes the B200 executable returned by
gnnc.compile.compile_executable. Sparse CSR inputs are decomposed into
(crow_indices, col_indices, values) exactly as the reference's
`_decompose_sparse` does (gnnc/execution/__init__.py:72-100); the B200 runtime
narrows the indices to int32 on the device.
"""

from __future__ import annotations

import torch

__all__ = ["run_jit"]


def run_jit(lowered, results: list, inputs: tuple) -> list[torch.Tensor]:
    """Invoke `lowered` on `inputs`; returns the outputs (host tensors for host inputs)."""
    from gnnc.b200.program import B200Executable

    if not isinstance(lowered, B200Executable):
        raise NotImplementedError(f"cannot run {type(lowered).__name__}: not a B200 executable")
    outs = lowered(*(t.detach() for t in inputs))
    if len(outs) != len(results):
        raise RuntimeError(f"executable returned {len(outs)} outputs, expected {len(results)}")
    return outs


def _decompose_sparse(args) -> list[torch.Tensor]:
    """Flattens inputs, expanding CSR into (crow_indices, col_indices, values)."""
    out = []
    for t in args:
        t = t.detach()
        if t.layout == torch.strided:
            out.append(t.contiguous())
        elif t.layout == torch.sparse_csr:
            out.extend([t.crow_indices().contiguous(), t.col_indices().contiguous(),
                        t.values().contiguous()])
        else:
            raise NotImplementedError(f"unsupported tensor layout: {t.layout}")
    return out
