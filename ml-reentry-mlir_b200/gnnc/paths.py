"""Host-side configurable paths (same variables as the reference's gnnc/paths.py:18-27)."""

from __future__ import annotations

import os
from pathlib import Path


def _resolve(env_var: str, fallback: Path) -> Path:
    value = os.environ.get(env_var)
    return Path(value) if value else fallback


DATA_DIR: Path = _resolve(
    "GNNC_DATA_DIR",
    Path(os.environ.get("XDG_DATA_HOME", str(Path.home() / ".local" / "share"))) / "gnnc",
)

CACHE_DIR: Path = _resolve(
    "GNNC_CACHE_DIR",
    Path(os.environ.get("XDG_CACHE_HOME", str(Path.home() / ".cache"))) / "gnnc",
)
