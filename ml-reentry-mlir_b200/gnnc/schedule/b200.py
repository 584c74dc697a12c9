"""The B200 lowering recipe: the phases that follow ingress for target="b200".

Takes the place of the reference's build_pipeline(target=...) (gnnc/schedule/sparse.py:21-114),
whose cpu/gpu branches run MLIR's sparsifier and, for gpu, NVVM codegen for sm_89.
Here the phases are:

  b200-lower : fx graph -> B200Program (GCNConv/GATConv chain, epilogue fusion)
  b200-bind  : B200Program -> B200Executable (weights on the device, feature dtype)
"""

from __future__ import annotations

import torch

from gnnc.pipeline.phase import PhasePipeline


def build_pipeline(
    *,
    target: str,
    feature_dtype: torch.dtype | None = None,
    output_dtype: torch.dtype | None = None,
    device=None,
) -> PhasePipeline:
    if target != "b200":
        raise NotImplementedError(f"target {target!r} not supported by this schedule")
    from gnnc.b200.program import B200Executable, lower_graph

    pipeline = PhasePipeline()
    pipeline.add_callable_phase(
        "b200-lower",
        lambda gm: lower_graph(gm, feature_dtype, output_dtype),
        ("match-conv-chain", "fuse-bias-activation", "fuse-log-softmax"),
    )
    pipeline.add_callable_phase(
        "b200-bind",
        lambda prog: B200Executable(prog, device),
        ("weights-to-device", "pad-rows-16B"),
    )
    return pipeline
