"""ctypes binding of libgnnc_b200.so (the C ABI declared in include/gnnc_b200.h).

The library is loaded from this directory, where `build_ext.py` (or `make` in
csrc/) puts it. There is no fallback: a missing or unloadable library raises
ImportError, which `gnnc-bench` maps to exit code 3 exactly like the reference
maps a missing MLIR stack (gnnc/tools/gnnc_bench.py:64-66).
"""

from __future__ import annotations

import ctypes
from ctypes import POINTER, c_char_p, c_float, c_int, c_int32, c_int64, c_size_t, c_void_p
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libgnnc_b200.so"

# gnnc_status_t
OK = 0
ERR_INVALID = 1
ERR_UNSUPPORTED = 2
ERR_CUDA = 3
ERR_OOM = 4
ERR_BOUNDS = 5
ERR_TIMEOUT = 6
ERR_NCCL = 7

# gnnc_dtype_t / gnnc_act_t
F32 = 0
BF16 = 1
ACT_NONE = 0
ACT_RELU = 1
ACT_ELU = 2

_P = c_void_p
_I64 = c_int64

# name -> (restype, argtypes); one line per declaration of include/gnnc_b200.h.
SIGNATURES: dict[str, tuple] = {
    "gnnc_init": (c_int, [c_int, POINTER(c_void_p)]),
    "gnnc_destroy": (c_int, [_P]),
    "gnnc_stream_set": (c_int, [_P, _P]),
    "gnnc_last_error": (c_int, [_P, c_char_p, c_size_t]),
    "gnnc_status_string": (c_char_p, [c_int]),
    "gnnc_abi_version": (c_int, []),
    "gnnc_synchronize": (c_int, [_P]),
    "gnnc_workspace_query": (c_int, [_P, _P, _I64, POINTER(c_size_t)]),
    "gnnc_workspace_bind": (c_int, [_P, _P, c_size_t]),
    "gnnc_csr_from_coo": (
        c_int,
        [_P, _P, _P, _I64, _I64, c_int, c_int, _P, _P, _P, _I64, POINTER(c_int64)],
    ),
    "gnnc_gcn_norm": (c_int, [_P, _P, _P, _P, _I64, _P, _P, _P]),
    "gnnc_csr_validate": (c_int, [_P, _P, _P, _I64, _I64, _I64]),
    "gnnc_plan_create": (c_int, [_P, _P, _I64, c_int32, c_int32, POINTER(c_void_p)]),
    "gnnc_plan_destroy": (c_int, [_P]),
    "gnnc_plan_info": (c_int, [_P, POINTER(c_int64)]),
    "gnnc_proj": (
        c_int,
        [_P, _P, c_int, _I64, _P, _I64, _I64, _I64, _I64, _P, _P, _I64, _P, c_int, _I64, _P, _P],
    ),
    "gnnc_gcn_aggregate": (
        c_int,
        [_P, _P, _P, _P, _P, _P, c_int, _I64, _I64, _I64, _I64, _P, c_int, c_int, _P, c_int, _I64],
    ),
    "gnnc_gat_aggregate": (
        c_int,
        [
            _P, _P, _P, _P, _P, c_int, _I64, _P, _P, _I64, _I64, _I64, _I64, c_float, c_int,
            _P, c_int, c_int, _P, c_int, _I64,
        ],
    ),
    "gnnc_mean_norm": (c_int, [_P, _P, _I64, _P, _P]),
    "gnnc_sage_aggregate": (
        c_int,
        [_P, _P, _P, _P, _P, _P, c_int, _I64, _P, c_int, _I64, _I64, _I64, _I64, _P, c_int,
         c_int, _P, c_int, _I64],
    ),
    "gnnc_peer_export": (c_int, [_P, _P, _P, POINTER(ctypes.c_uint64)]),
    "gnnc_peer_open": (c_int, [_P, _P, ctypes.c_uint64, POINTER(c_void_p)]),
    "gnnc_peer_close": (c_int, [_P, _P, ctypes.c_uint64]),
    "gnnc_peer_copy": (c_int, [_P, _P, _P, c_size_t]),
    "gnnc_gather_rows": (c_int, [_P, _P, _I64, _P, _I64, _I64, _P, _I64, _I64]),
    "gnnc_comm_unique_id": (c_int, [_P, _P]),
    "gnnc_comm_init": (c_int, [_P, _P, c_int, c_int]),
    "gnnc_comm_init_timeout": (c_int, [_P, _P, c_int, c_int, _I64]),
    "gnnc_allgather": (c_int, [_P, _P, _P, c_size_t, c_int]),
    "gnnc_comm_wait": (c_int, [_P, _I64]),
    "gnnc_wait_selftest": (c_int, [_P, _I64]),
    "gnnc_comm_destroy": (c_int, [_P]),
    "gnnc_gat_aggregate_noalloc": (
        c_int,
        [
            _P, _P, _P, _P, _P, c_int, _I64, _P, _P, _I64, _I64, _I64, _I64, c_float, c_int,
            _P, c_int, c_int, _P, c_int, _I64,
        ],
    ),
    "gnnc_softmax_aggregate": (
        c_int,
        [
            _P, _P, _P, _P, _P, _P, c_int, _I64, _I64, _I64, _I64, _I64, c_float, c_int, _P,
            c_int, c_int, _P, c_int, _I64,
        ],
    ),
}


class GnncError(RuntimeError):
    """A non-zero gnnc_status_t; `status` holds the code."""

    def __init__(self, status: int, message: str) -> None:
        super().__init__(message)
        self.status = status


class GnncInvalidArgument(GnncError, ValueError):
    """GNNC_ERR_INVALID / GNNC_ERR_BOUNDS: maps to gnnc-bench exit code 2."""


class GnncUnsupported(GnncError, NotImplementedError):
    """GNNC_ERR_UNSUPPORTED: maps to gnnc-bench exit code 2."""


_lib: ctypes.CDLL | None = None


def load() -> ctypes.CDLL:
    """Loads (once) and returns the library with every signature bound."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise ImportError(
            f"libgnnc_b200.so not built ({LIB_PATH}); run `python ml-reentry-mlir_b200/build_ext.py`"
        )
    try:
        lib = ctypes.CDLL(str(LIB_PATH))
    except OSError as exc:  # pragma: no cover - depends on the system loader
        raise ImportError(f"cannot load {LIB_PATH}: {exc}") from exc
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def raise_for(status: int, ctx: int | None, what: str) -> None:
    """Raises the exception matching `status` with the context's error text."""
    if status == OK:
        return
    lib = load()
    text = ""
    if ctx:
        buf = ctypes.create_string_buffer(1024)
        lib.gnnc_last_error(ctx, buf, len(buf))
        text = buf.value.decode(errors="replace")
    kind = lib.gnnc_status_string(status).decode()
    msg = f"{what}: {kind}" + (f": {text}" if text else "")
    if status in (ERR_INVALID, ERR_BOUNDS):
        raise GnncInvalidArgument(status, msg)
    if status == ERR_UNSUPPORTED:
        raise GnncUnsupported(status, msg)
    raise GnncError(status, msg)
