"""End-to-end compile pipeline: torch model -> B200 executable.

Same two entry points as the reference's gnnc/compile.py:127-208:

- `lower(model, inputs, ...)` runs the phase pipeline (import -> b200-lower ->
  b200-bind), halting where asked, and returns `(module, trace)`.
- `compile_executable(model, inputs, target=...)` runs it to the end and
  returns `(lowered, results)` ready for `gnnc.execution.run_jit`.

Only target="b200" is built here. The reference's "cpu" and "gpu" targets are
MLIR pipelines (torch-mlir + Lighthouse + the sparsifier); asking for them
raises ImportError, which gnnc-bench reports with exit code 3 just as the
reference does when its MLIR stack is missing (gnnc/tools/gnnc_bench.py:64-66).
"""

from __future__ import annotations

import torch

from gnnc import get_context
from gnnc.pipeline.phase import PhasePipeline
from gnnc.schedule.b200 import build_pipeline

__all__ = ["compile_executable", "lower"]

_MLIR_TARGETS = ("cpu", "gpu")


def _check_target(target: str) -> None:
    if target in _MLIR_TARGETS:
        raise ImportError(
            f"target {target!r} is the reference's MLIR pipeline (torch-mlir, Lighthouse); "
            "this build provides target='b200'"
        )
    if target != "b200":
        raise NotImplementedError(f"target {target!r} not supported")


def _feature_dtype(forward_inputs: tuple, dtype) -> torch.dtype:
    if dtype is not None:
        return {"fp32": torch.float32, "bf16": torch.bfloat16}.get(dtype, dtype)
    x = forward_inputs[0]
    return torch.bfloat16 if x.dtype == torch.bfloat16 else torch.float32


def _frontend_pipeline(model: torch.nn.Module) -> PhasePipeline:
    from gnnc.b200.program import trace

    pipeline = PhasePipeline()
    pipeline.add_callable_phase("import", lambda _: trace(model), ("torch.fx trace (convs as leaves)",))
    return pipeline


def lower(
    model: torch.nn.Module,
    forward_inputs: tuple,
    *,
    target: str = "b200",
    stop_before: str | None = None,
    stop_after: str | None = None,
    print_ir_before: frozenset[str] = frozenset(),
    print_ir_after: frozenset[str] = frozenset(),
    emit=print,
    dtype=None,
    out_dtype=None,
    device=None,
):
    """Run the phase pipeline, halting per `stop_*`. Returns `(module, trace)`.

    dtype: feature dtype on the device ("fp32" / "bf16" / torch dtype; default
    the input's); out_dtype: dtype of the returned output (default float32)."""
    _check_target(target)
    pipeline = _frontend_pipeline(model)
    pipeline.extend(
        build_pipeline(
            target=target,
            feature_dtype=_feature_dtype(forward_inputs, dtype),
            output_dtype=_feature_dtype(forward_inputs, out_dtype) if out_dtype else None,
            device=device,
        )
    )
    return pipeline.run(
        None,
        get_context,
        stop_before=stop_before,
        stop_after=stop_after,
        print_ir_before=print_ir_before,
        print_ir_after=print_ir_after,
        emit=emit,
    )


def compile_executable(
    model: torch.nn.Module,
    forward_inputs: tuple,
    *,
    target: str = "b200",
    dtype=None,
    out_dtype=None,
    device=None,
):
    """Compile `model` for `target`; returns `(lowered, results)`.

    `lowered` is a B200Executable; `results` lists the output's (shape, dtype),
    the analogue of the entry function's result types in the reference."""
    lowered, _ = lower(model, forward_inputs, target=target, dtype=dtype, out_dtype=out_dtype,
                       device=device)
    n = forward_inputs[0].size(0)
    width = lowered.program.layers[-1].out_width
    return lowered, [((n, width), lowered.program.output_dtype)]
