"""Reference models and example data (KernelBench convention: Model,
get_init_inputs(), get_inputs()), as in the reference's gnnc/examples/__init__.py:1-20."""

from __future__ import annotations

from pathlib import Path

MODELS_DIR = Path(__file__).parent / "models"

__all__ = ["MODELS_DIR", "available"]


def available() -> list[str]:
    """Model names (file stems) discoverable in `models/`."""
    return sorted(p.stem for p in MODELS_DIR.glob("*.py") if not p.stem.startswith("_"))
