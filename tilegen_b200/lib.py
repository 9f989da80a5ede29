"""ctypes binding of libtilegen_b200.so (declarations in include/tilegen_b200.h).

The library is looked up in ``$TILEGEN_B200_LIB`` or next to this file (built in-tree
by ``python -m tilegen_b200.build``).  There is no fallback: if the library cannot be
loaded every entry point raises :class:`LibraryError`.
"""

from __future__ import annotations

import ctypes
import os
import re
from typing import List, Optional

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
REPO_DIR = os.path.dirname(PKG_DIR)
HEADER = os.path.join(REPO_DIR, "include", "tilegen_b200.h")

TG_OK = 0
TG_EINVAL = -1
TG_ECUDA = -2
TG_ENOMEM = -3
TG_EUNSUPPORTED = -4
TG_ETIMEDOUT = -5
TG_EBOUNDS = -6

TG_SPLIT_ROWWISE = 0
TG_SPLIT_MERGE = 1
TG_SPLIT_AUTO = 2
TG_SPLIT_STREAM = 3
TG_SPLIT_BLOCK = 4

TG_FLAG_BOUNDS_CHECK = 1
TG_FLAG_INJECT_BUG = 2
TG_FLAG_REUSE_PLAN = 4
TG_FLAG_INDEX32 = 8

STATUS_NAMES = {
    TG_OK: "TG_OK",
    TG_EINVAL: "TG_EINVAL",
    TG_ECUDA: "TG_ECUDA",
    TG_ENOMEM: "TG_ENOMEM",
    TG_EUNSUPPORTED: "TG_EUNSUPPORTED",
    TG_ETIMEDOUT: "TG_ETIMEDOUT",
    TG_EBOUNDS: "TG_EBOUNDS",
}


class LibraryError(RuntimeError):
    """libtilegen_b200.so is missing or failed to load."""


class TgError(RuntimeError):
    """A tg_* call returned a negative status."""

    def __init__(self, status: int, what: str, message: str):
        self.status = status
        super().__init__("%s failed: %s (%s)" % (what, STATUS_NAMES.get(status, status), message))


class TgSched(ctypes.Structure):
    _fields_ = [
        ("tile", ctypes.c_int32),
        ("threads_per_row", ctypes.c_int32),
        ("unroll", ctypes.c_int32),
        ("vector_width", ctypes.c_int32),
        ("block_size", ctypes.c_int32),
        ("split", ctypes.c_int32),
        ("chunk_nnz", ctypes.c_int32),
        ("flags", ctypes.c_uint32),
    ]

    def as_dict(self):
        return {name: getattr(self, name) for name, _ in self._fields_}


class TgCsr(ctypes.Structure):
    _fields_ = [
        ("rows", ctypes.c_int64),
        ("cols", ctypes.c_int64),
        ("nnz", ctypes.c_int64),
        ("indptr", ctypes.c_void_p),
        ("indices", ctypes.c_void_p),
        ("data", ctypes.c_void_p),
    ]


_I64 = ctypes.c_int64
_P = ctypes.c_void_p
_F64 = ctypes.c_double
_SZ = ctypes.c_size_t
_SP = ctypes.POINTER(TgSched)
_CP = ctypes.POINTER(TgCsr)

# name -> (restype, argtypes); every symbol declared in include/tilegen_b200.h
SIGNATURES = {
    "tg_version": (ctypes.c_char_p, []),
    "tg_last_error_string": (ctypes.c_char_p, []),
    "tg_last_status": (ctypes.c_int, []),
    "tg_launch_count": (ctypes.c_uint64, []),
    "tg_dist_init": (ctypes.c_int, [ctypes.c_int32, ctypes.POINTER(ctypes.c_int32), ctypes.POINTER(ctypes.c_void_p)]),
    "tg_dist_finalize": (ctypes.c_int, [ctypes.c_void_p]),
    "tg_dist_spmv_power": (ctypes.c_int, [ctypes.c_void_p, _CP, ctypes.c_void_p, ctypes.c_int32, _SP, ctypes.c_void_p,
                                          ctypes.c_void_p, ctypes.c_double]),
    "tg_dist_spmm_f32": (ctypes.c_int, [ctypes.c_void_p, _CP, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, _SP,
                                        ctypes.c_double]),
    "tg_dist_sddmm_f32": (ctypes.c_int, [ctypes.c_void_p, _CP, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64,
                                         ctypes.c_void_p, _SP, ctypes.c_double]),
    "tg_renumber_columns": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p,
                                           ctypes.c_int32, ctypes.c_int64, ctypes.c_void_p]),
    "tg_renumber_columns_i32": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p,
                                               ctypes.c_int32, ctypes.c_int64, ctypes.c_void_p]),
    "tg_default_schedule": (None, [_SP]),
    "tg_validate_schedule": (ctypes.c_int, [_SP]),
    "tg_set_schedule": (ctypes.c_int, [_SP]),
    "tg_get_schedule": (ctypes.c_int, [_SP]),
    "tg_spmv_workspace_bytes": (_SZ, [_I64, _I64, _SP]),
    "tg_spmm_workspace_bytes": (_SZ, [_I64, _I64, _I64, _SP]),
    "tg_sddmm_workspace_bytes": (_SZ, [_I64, _I64, _I64, _SP]),
    "tg_spmv_f64": (ctypes.c_int, [_CP, _P, _P, _SP, _P, _SZ, _P]),
    "tg_spmv_f32": (ctypes.c_int, [_CP, _P, _P, _SP, _P, _SZ, _P]),
    "tg_fused_spmv_axpy_f64": (ctypes.c_int, [_CP, _P, _P, _P, _F64, _F64, _SP, _P, _SZ, _P]),
    "tg_fused_spmv_axpy_f32": (ctypes.c_int, [_CP, _P, _P, _P, ctypes.c_float, ctypes.c_float, _SP, _P, _SZ, _P]),
    "tg_spmm_f32": (ctypes.c_int, [_CP, _P, _P, _I64, _SP, _P, _SZ, _P]),
    "tg_spmm_f64": (ctypes.c_int, [_CP, _P, _P, _I64, _SP, _P, _SZ, _P]),
    "tg_sddmm_f32": (ctypes.c_int, [_CP, _P, _P, _P, _I64, _SP, _P, _SZ, _P]),
    "tg_sddmm_f64": (ctypes.c_int, [_CP, _P, _P, _P, _I64, _SP, _P, _SZ, _P]),
    "tg_axpy_f64": (ctypes.c_int, [_P, _P, _P, _F64, _F64, _I64, _SP, _P]),
    "tg_axpy_f32": (ctypes.c_int, [_P, _P, _P, ctypes.c_float, ctypes.c_float, _I64, _SP, _P]),
    "tg_power_workspace_bytes": (_SZ, [_I64, _SP]),
    "tg_power_step_f64": (ctypes.c_int, [_CP, _P, ctypes.c_int32, _I64, _P, _SP, _P, _SZ, _P]),
    "tg_shard_norm2_f64": (ctypes.c_int, [_P, _I64, _I64, _P, _SZ, _P]),
    "tg_power_finalize_f64": (ctypes.c_int, [_P, ctypes.c_int32, _I64, ctypes.c_int32, _I64, _P, _P, _P]),
    "tg_power_step_p2p_f64": (ctypes.c_int, [_CP, _P, ctypes.c_int32, ctypes.c_int32, _I64, _P, _P,
                                             ctypes.c_uint64, _SP, _P, _SZ, _P]),
    "tg_p2p_wait": (ctypes.c_int, [_P, ctypes.c_int32, ctypes.c_uint64, _P, _SZ, _P]),
    "tg_power_error": (ctypes.c_int, [_P, ctypes.POINTER(ctypes.c_uint32), _P]),
    "tg_power_clear_error": (ctypes.c_int, [_P, _P]),
    "tg_power_step_ce_f64": (ctypes.c_int, [_CP, _P, ctypes.c_int32, ctypes.c_int32, _I64, _P, _P, ctypes.c_uint64,
                                            ctypes.c_int32, _SP, _P, _SZ, _P]),
    "tg_peer_buffer_alloc": (ctypes.c_int, [_SZ, ctypes.POINTER(ctypes.c_void_p)]),
    "tg_peer_buffer_free": (ctypes.c_int, [_P]),
    "tg_ipc_get_handle": (ctypes.c_int, [_P, ctypes.c_char_p]),
    "tg_ipc_open": (ctypes.c_int, [ctypes.c_char_p, ctypes.POINTER(ctypes.c_void_p)]),
    "tg_ipc_close": (ctypes.c_int, [_P]),
    "tg_spmv_f64_noalloc": (ctypes.c_int, [_CP, _P, _P, _SP, _P]),
    "tg_rcm_order": (ctypes.c_int, [_I64, _P, _P, _P]),
    "launch_spmv": (None, [_P, _P, _P, _P, _P, _I64, _I64, _I64]),
    "launch_spmm": (None, [_P, _P, _P, _P, _P, _I64, _I64, _I64, _I64]),
    "launch_sddmm": (None, [_P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64]),
    "launch_fused_spmv_axpy": (None, [_P, _P, _P, _P, _P, _P, _F64, _F64, _I64, _I64, _I64]),
    "launch_axpy": (None, [_P, _P, _P, _F64, _F64, _I64]),
}

_lib: Optional[ctypes.CDLL] = None


def lib_path() -> str:
    env = os.environ.get("TILEGEN_B200_LIB")
    if env:
        return env
    return os.path.join(PKG_DIR, "libtilegen_b200.so")


def load() -> ctypes.CDLL:
    """Load (once) and type the library; raises LibraryError when it is absent."""
    global _lib
    if _lib is not None:
        return _lib
    path = lib_path()
    if not os.path.exists(path):
        raise LibraryError("libtilegen_b200.so not found at %s; build it with `python -m tilegen_b200.build` "
                           "(there is no CPU fallback)" % path)
    try:
        L = ctypes.CDLL(path)
    except OSError as exc:
        raise LibraryError("cannot load %s: %s" % (path, exc)) from exc
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def header_symbols(path: str = HEADER) -> List[str]:
    """Function names declared in include/tilegen_b200.h."""
    text = open(path).read()
    return re.findall(r"^TG_API\s+[\w\s\*]+?\b(\w+)\s*\(", text, flags=re.M)


def last_error() -> str:
    msg = load().tg_last_error_string()
    return msg.decode("utf-8", "replace") if msg else ""


def check(status: int, what: str) -> None:
    if status != TG_OK:
        raise TgError(status, what, last_error())


def version() -> str:
    return load().tg_version().decode()


def default_schedule() -> TgSched:
    s = TgSched()
    load().tg_default_schedule(ctypes.byref(s))
    return s


def validate_schedule(s: TgSched) -> None:
    check(load().tg_validate_schedule(ctypes.byref(s)), "tg_validate_schedule")


def set_schedule(s: TgSched) -> None:
    check(load().tg_set_schedule(ctypes.byref(s)), "tg_set_schedule")


def get_schedule() -> TgSched:
    s = TgSched()
    check(load().tg_get_schedule(ctypes.byref(s)), "tg_get_schedule")
    return s
