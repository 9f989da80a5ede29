"""ctypes front end of the parity oracle (TEST INFRASTRUCTURE ONLY).

Loads ``oracle/_build/liboracle.so`` (the C restatement in ``tg_oracle.c``, built on
demand) and, when present, the reference-compiled checkers in ``oracle/_ref/``:
``libtgref.so`` (the reference's serial ``cpp/src/ref.cpp``) and the reference's
OpenMP-emitted ``launch_<kernel>`` objects.  Only tests, ``__graft_entry__.smoke()`` and
the CPU legs of ``bench.py`` may use this module; it is the checker, never the product.

All functions take/return numpy arrays; CSR arguments are ``(indptr, indices, data)``
with int64 index arrays.
"""

from __future__ import annotations

import ctypes
import glob
import json
import os
from typing import Dict, Optional, Tuple

import numpy as np

from . import build as _build

I64 = ctypes.c_int64
F64 = ctypes.c_double
P = ctypes.c_void_p

_lib: Optional[ctypes.CDLL] = None
_ref: Optional[ctypes.CDLL] = None


def _ptr(a: np.ndarray) -> ctypes.c_void_p:
    return ctypes.c_void_p(a.ctypes.data)


def lib() -> ctypes.CDLL:
    """The C oracle (built if missing)."""
    global _lib
    if _lib is None:
        path = _build.ORACLE_LIB
        if not os.path.exists(path):
            path = _build.build_oracle()
        L = ctypes.CDLL(path)
        for name in ("tgo_spmv_f64", "tgo_spmv_f32"):
            getattr(L, name).argtypes = [P, P, P, P, P, I64]
        L.tgo_spmv_rows_f64.argtypes = [P, P, P, P, P, I64, I64]
        L.tgo_spmv_f64_omp.argtypes = [P, P, P, P, P, I64]
        L.tgo_spmv_f64_omp.restype = ctypes.c_int
        for name in ("tgo_spmm_f64", "tgo_spmm_f32"):
            getattr(L, name).argtypes = [P, P, P, P, P, I64, I64]
        for name in ("tgo_sddmm_f64", "tgo_sddmm_f32"):
            getattr(L, name).argtypes = [P, P, P, P, P, P, I64, I64]
        L.tgo_fused_spmv_axpy_f64.argtypes = [P, P, P, P, P, P, F64, F64, I64]
        L.tgo_axpy_f64.argtypes = [P, P, P, F64, F64, I64]
        L.tgo_power_iteration_f64.argtypes = [P, P, P, P, P, I64, ctypes.c_int]
        L.tgo_power_iteration_f64.restype = F64
        _lib = L
    return _lib


def _csr(A, vdtype) -> Tuple[np.ndarray, np.ndarray, np.ndarray, int]:
    if hasattr(A, "indptr"):
        ip, ix, d = A.indptr, A.indices, A.data
    else:
        ip, ix, d = A
    ip = np.ascontiguousarray(ip, dtype=np.int64)
    ix = np.ascontiguousarray(ix, dtype=np.int64)
    d = np.ascontiguousarray(d, dtype=vdtype)
    return ip, ix, d, ip.size - 1


def spmv(A, x: np.ndarray, dtype=np.float64) -> np.ndarray:
    ip, ix, d, rows = _csr(A, dtype)
    x = np.ascontiguousarray(x, dtype=dtype)
    y = np.empty(rows, dtype=dtype)
    fn = lib().tgo_spmv_f64 if dtype == np.float64 else lib().tgo_spmv_f32
    fn(_ptr(ip), _ptr(ix), _ptr(d), _ptr(x), _ptr(y), rows)
    return y


def spmv_rows(A, x: np.ndarray, r0: int, r1: int) -> np.ndarray:
    """Rows [r0, r1) of A x (fp64); A may be any (indptr, indices, data) view."""
    ip, ix, d, _ = _csr(A, np.float64)
    x = np.ascontiguousarray(x, dtype=np.float64)
    y = np.empty(max(r1 - r0, 0), dtype=np.float64)
    lib().tgo_spmv_rows_f64(_ptr(ip), _ptr(ix), _ptr(d), _ptr(x), _ptr(y), r0, r1)
    return y


def spmv_omp(A, x: np.ndarray, out: Optional[np.ndarray] = None) -> Tuple[np.ndarray, int]:
    """Multi-threaded fp64 SpMV (the 'port' CPU baseline); returns (y, threads used)."""
    ip, ix, d, rows = _csr(A, np.float64)
    x = np.ascontiguousarray(x, dtype=np.float64)
    y = out if out is not None else np.empty(rows, dtype=np.float64)
    n = lib().tgo_spmv_f64_omp(_ptr(ip), _ptr(ix), _ptr(d), _ptr(x), _ptr(y), rows)
    return y, int(n)


def spmm(A, B: np.ndarray, dtype=np.float64) -> np.ndarray:
    ip, ix, d, rows = _csr(A, dtype)
    B = np.ascontiguousarray(B, dtype=dtype)
    K = B.shape[1]
    C = np.empty((rows, K), dtype=dtype)
    fn = lib().tgo_spmm_f64 if dtype == np.float64 else lib().tgo_spmm_f32
    fn(_ptr(ip), _ptr(ix), _ptr(d), _ptr(B), _ptr(C), rows, K)
    return C


def sddmm(A, U: np.ndarray, V: np.ndarray, dtype=np.float64) -> np.ndarray:
    ip, ix, d, rows = _csr(A, dtype)
    U = np.ascontiguousarray(U, dtype=dtype)
    V = np.ascontiguousarray(V, dtype=dtype)
    K = U.shape[1]
    out = np.empty(ix.size, dtype=dtype)
    fn = lib().tgo_sddmm_f64 if dtype == np.float64 else lib().tgo_sddmm_f32
    fn(_ptr(ip), _ptr(ix), _ptr(d), _ptr(U), _ptr(V), _ptr(out), rows, K)
    return out


def fused_spmv_axpy(A, x, w, alpha: float, beta: float) -> np.ndarray:
    ip, ix, d, rows = _csr(A, np.float64)
    x = np.ascontiguousarray(x, dtype=np.float64)
    w = np.ascontiguousarray(w, dtype=np.float64)
    z = np.empty(rows, dtype=np.float64)
    lib().tgo_fused_spmv_axpy_f64(_ptr(ip), _ptr(ix), _ptr(d), _ptr(x), _ptr(w), _ptr(z), alpha, beta, rows)
    return z


def axpy(x, w, alpha: float, beta: float) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float64)
    w = np.ascontiguousarray(w, dtype=np.float64)
    z = np.empty_like(x)
    lib().tgo_axpy_f64(_ptr(x), _ptr(w), _ptr(z), alpha, beta, x.size)
    return z


def power_iteration(A, x0: np.ndarray, iters: int) -> Tuple[np.ndarray, float]:
    """x <- A x / ||A x|| `iters` times (fp64); returns (x, last norm)."""
    ip, ix, d, rows = _csr(A, np.float64)
    x = np.array(x0, dtype=np.float64, copy=True)
    y = np.empty(rows, dtype=np.float64)
    nrm = lib().tgo_power_iteration_f64(_ptr(ip), _ptr(ix), _ptr(d), _ptr(x), _ptr(y), rows, iters)
    return x, float(nrm)


# ------------------------------------------------------------------ reference builds
def ref_lib() -> Optional[ctypes.CDLL]:
    """The reference's serial C++ kernels (oracle/_ref/libtgref.so), if built."""
    global _ref
    if _ref is None and os.path.exists(_build.TGREF_LIB):
        L = ctypes.CDLL(_build.TGREF_LIB)
        for name in ("tgref_spmv_f64", "tgref_spmv_f32"):
            getattr(L, name).argtypes = [P, P, P, I64, I64, I64, P, P]
        for name in ("tgref_spmm_f64", "tgref_spmm_f32"):
            getattr(L, name).argtypes = [P, P, P, I64, I64, I64, P, I64, P]
        for name in ("tgref_sddmm_f64", "tgref_sddmm_f32"):
            getattr(L, name).argtypes = [P, P, P, I64, I64, I64, P, P, I64, P]
        L.tgref_fused_spmv_axpy_f64.argtypes = [P, P, P, I64, I64, I64, P, P, F64, F64, P]
        L.tgref_dense_spmv_f64.argtypes = [P, I64, I64, P, P]
        _ref = L
    return _ref


def ref_omp_libs(directory: Optional[str] = None) -> Dict[str, str]:
    """{stem: path} of the reference OpenMP launchers (``ref_omp_<kernel>_<dtype>_<cfg>``)."""
    directory = directory or _build.REF_DIR
    return {os.path.basename(p)[:-3]: p for p in sorted(glob.glob(os.path.join(directory, "ref_omp_*.so")))}


def ref_omp_manifest() -> Dict[str, dict]:
    path = os.path.join(_build.REF_DIR, "manifest.json")
    if not os.path.exists(path):
        return {}
    with open(path) as fh:
        return json.load(fh)


class RefOmpKernel:
    """A reference OpenMP ``launch_<kernel>`` called on host buffers, with the argument
    order of tilegen/verify.py:166-173 (``float*`` instead of ``double*`` for f32)."""

    def __init__(self, path: str, kernel: str, dtype: str = "f64"):
        self.path = path
        self.kernel = kernel
        self.lib = ctypes.CDLL(path)
        self.fn = getattr(self.lib, "launch_%s" % kernel)
        # the scalars alpha/beta have the kernel's dtype (tilegen/codegen.py:270-271)
        S = F64 if dtype == "f64" else ctypes.c_float
        nptr = {"spmv": 5, "spmm": 5, "sddmm": 6, "fused_spmv_axpy": 6, "axpy": 3}[kernel]
        tail = {"spmv": [I64] * 3, "spmm": [I64] * 4, "sddmm": [I64] * 4,
                "fused_spmv_axpy": [S, S, I64, I64, I64], "axpy": [S, S, I64]}[kernel]
        self.fn.argtypes = [P] * nptr + tail
        self.fn.restype = None

    def __call__(self, *args):
        conv = [_ptr(a) if isinstance(a, np.ndarray) else a for a in args]
        self.fn(*conv)
