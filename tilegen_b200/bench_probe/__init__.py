"""The benchmark's gather-floor probes (libtg_gather_probe.so): the random x gathers of a
CSR SpMV, or the dense-row gathers of an SpMM / SDDMM, and nothing else.  A measurement
aid, kept out of libtilegen_b200.so."""

from __future__ import annotations

import ctypes
import os
from typing import Optional

PROBE_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libtg_gather_probe.so")

_probe: Optional[ctypes.CDLL] = None


def load() -> ctypes.CDLL:
    """Load and type libtg_gather_probe.so (built by tilegen_b200.build)."""
    global _probe
    if _probe is None:
        if not os.path.exists(PROBE_PATH):
            raise OSError("libtg_gather_probe.so not found at %s; run `python -m tilegen_b200.build`" % PROBE_PATH)
        L = ctypes.CDLL(PROBE_PATH)
        for name in ("tg_gather_probe_f64", "tg_gather_probe_i32_f64"):
            fn = getattr(L, name)
            fn.restype = ctypes.c_int
            fn.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
        L.tg_row_gather_probe_f32.restype = ctypes.c_int
        L.tg_row_gather_probe_f32.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64,
                                              ctypes.c_void_p, ctypes.c_void_p]
        _probe = L
    return _probe


def gather_probe_f64(indices_ptr: int, n: int, x_ptr: int, out_ptr: int, stream: int, index32: bool = False) -> None:
    """*out += sum of x[indices[i]] for i < n, on `stream` (device pointers; int64 column
    indices, or int32 with ``index32``)."""
    L = load()
    fn = L.tg_gather_probe_i32_f64 if index32 else L.tg_gather_probe_f64
    rc = fn(indices_ptr, n, x_ptr, out_ptr, stream)
    if rc != 0:
        raise RuntimeError("tg_gather_probe_f64 failed with status %d" % rc)


def row_gather_probe_f32(indices_ptr: int, n: int, B_ptr: int, K: int, out_ptr: int, stream: int) -> None:
    """*out += sum of B[indices[i], :] for i < n, on `stream` (device pointers; int64
    indices; B row-major fp32 with K = 64 or 128 columns, 16-byte aligned)."""
    rc = load().tg_row_gather_probe_f32(indices_ptr, n, B_ptr, K, out_ptr, stream)
    if rc != 0:
        raise RuntimeError("tg_row_gather_probe_f32 failed with status %d" % rc)
