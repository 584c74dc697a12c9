"""Named compile phases (see gnnc.pipeline.phase)."""
