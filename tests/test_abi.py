"""The C-ABI library loads and exports every entry point include/gnnc_b200.h declares."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

from conftest import ROOT

HEADER = ROOT / "include" / "gnnc_b200.h"


def declared_symbols() -> list[str]:
    text = HEADER.read_text()
    return re.findall(r"^GNNC_API\s+[\w\s\*]+?\b(gnnc_\w+)\s*\(", text, flags=re.M)


def test_header_declares_entry_points():
    names = declared_symbols()
    assert len(names) >= 19
    assert len(set(names)) == len(names)


def test_library_exports_every_declared_symbol():
    from gnnc.b200 import _lib

    lib = _lib.load()
    missing = [n for n in declared_symbols() if not hasattr(lib, n)]
    assert not missing, missing


def test_bindings_cover_every_declaration():
    from gnnc.b200 import _lib

    assert set(declared_symbols()) == set(_lib.SIGNATURES)


def test_abi_version_and_status_strings():
    from gnnc.b200 import _lib

    lib = _lib.load()
    assert lib.gnnc_abi_version() == 1
    assert lib.gnnc_status_string(0) == b"ok"
    assert lib.gnnc_status_string(5) == b"index out of bounds"
    assert lib.gnnc_status_string(99) == b"unknown status"


def test_null_arguments_are_rejected_without_a_device():
    """Argument checks run before any CUDA call; nothing aborts."""
    from gnnc.b200 import _lib

    lib = _lib.load()
    assert lib.gnnc_init(0, None) == _lib.ERR_INVALID
    assert lib.gnnc_stream_set(None, None) == _lib.ERR_INVALID
    assert lib.gnnc_synchronize(None) == _lib.ERR_INVALID
    assert lib.gnnc_plan_info(None, None) == _lib.ERR_INVALID
    assert lib.gnnc_destroy(None) == _lib.OK
    assert lib.gnnc_comm_unique_id(None, None) == _lib.ERR_INVALID
    assert lib.gnnc_comm_init(None, None, 0, 1) == _lib.ERR_INVALID
    assert lib.gnnc_allgather(None, None, None, 0, 0) == _lib.ERR_INVALID
    assert lib.gnnc_comm_destroy(None) == _lib.ERR_INVALID
    assert lib.gnnc_comm_init_timeout(None, None, 0, 1, 1000) == _lib.ERR_INVALID
    assert lib.gnnc_comm_wait(None, 1000) == _lib.ERR_INVALID
    assert lib.gnnc_wait_selftest(None, 1000) == _lib.ERR_INVALID
    assert lib.gnnc_plan_destroy(None) == _lib.OK


def test_library_is_sm100a_only():
    """The shared object carries sm_100a code (checked from the ELF note names only)."""
    from gnnc.b200 import _lib

    data = Path(_lib.LIB_PATH).read_bytes()
    assert b"sm_100a" in data
    assert ctypes.sizeof(ctypes.c_void_p) == 8
