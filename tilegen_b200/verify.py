"""Differential verification of the b200 kernels (mirror of tilegen/verify.py).

``verify(kernel_name, config, matrix)`` builds the same inputs as the reference
(``inputs_for``: seed 7, x/w/B/U/V standard normal, alpha 0.7, beta -1.3;
tilegen/verify.py:338-347), computes the same SciPy float64 expectation
(``reference``; tilegen/verify.py:350-371), runs the b200 kernel through the C ABI on
device buffers and applies the reference's acceptance rule
``max_abs <= 8 * eps * max_row_nnz * max|ref| + 1e-12`` (tilegen/verify.py:510-514),
with eps of the compute dtype.  Like the reference it also reports the max relative
error (floored denominator, tilegen/verify.py:507).

``run_launcher`` drives the reference-compatible ``launch_<name>`` entry points of the
library exactly as the reference's ``run_kernel`` drives a generated CUDA .so: device
buffers, one call, synchronize, copy back (tilegen/verify.py:414-451).
"""

from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass, field
from typing import Any, Dict, Sequence, Tuple

import numpy as np

from . import codegen as _codegen
from . import lib as _lib
from .matrices import CSR

__all__ = ["VerifyResult", "verify", "inputs_for", "reference", "load_matrix", "run_kernel", "run_launcher",
           "tolerance"]

KERNELS = ("spmv", "spmm", "sddmm", "fused_spmv_axpy", "axpy")


def load_matrix(matrix) -> Tuple[CSR, str]:
    """npz path (tilegen/matrices.py:215-237 layout), dict, scipy matrix or CSR."""
    if isinstance(matrix, CSR):
        return matrix, matrix.name
    if isinstance(matrix, str):
        with np.load(matrix, allow_pickle=False) as z:
            name = str(z["class_name"]) if "class_name" in z else os.path.basename(matrix)
            return CSR(z["indptr"].astype(np.int64), z["indices"].astype(np.int64), z["data"].astype(np.float64),
                       tuple(int(s) for s in z["shape"]), name), name
    if isinstance(matrix, dict):
        m = CSR(np.asarray(matrix["indptr"], np.int64), np.asarray(matrix["indices"], np.int64),
                np.asarray(matrix["data"], np.float64), tuple(matrix["shape"]), matrix.get("class_name", "custom"))
        return m, m.name
    if hasattr(matrix, "tocsr"):
        m = CSR.from_scipy(matrix.tocsr().astype(np.float64), "custom")
        return m, "custom"
    raise TypeError("unsupported matrix type: %r" % type(matrix))


def inputs_for(kernel: str, A: CSR, K: int, seed: int = 7):
    """x (N), w (M), B (N,K), U (M,K), V (N,K) ~ N(0,1) in that draw order, alpha 0.7,
    beta -1.3 (tilegen/verify.py:338-347)."""
    M, N = A.shape
    rng = np.random.default_rng(seed)
    x = rng.standard_normal(N)
    w = rng.standard_normal(M)
    B = rng.standard_normal((N, K))
    U = rng.standard_normal((M, K))
    V = rng.standard_normal((N, K))
    return x, w, B, U, V, 0.7, -1.3


def reference(kernel: str, A: CSR, data) -> np.ndarray:
    """SciPy float64 expectation (tilegen/verify.py:350-371)."""
    x, w, B, U, V, alpha, beta = data
    S = A.to_scipy().astype(np.float64)
    if kernel == "spmv":
        return np.asarray(S @ x, dtype=np.float64)
    if kernel == "spmm":
        return np.asarray(S @ B, dtype=np.float64)
    if kernel == "sddmm":
        rows = np.repeat(np.arange(A.rows, dtype=np.int64), np.diff(A.indptr))
        out = np.empty(A.nnz, dtype=np.float64)
        step = 200000
        for s in range(0, A.nnz, step):
            e = min(s + step, A.nnz)
            out[s:e] = np.einsum("ik,ik->i", U[rows[s:e]], V[A.indices[s:e]]) * A.data[s:e]
        return out
    if kernel == "fused_spmv_axpy":
        return alpha * (S @ x) + beta * w
    if kernel == "axpy":
        return alpha * x + beta * w
    raise ValueError("unknown kernel %r" % kernel)


def tolerance(A: CSR, refv: np.ndarray, dtype: str = "f64") -> float:
    eps = float(np.finfo(np.float64 if dtype == "f64" else np.float32).eps)
    scale = float(np.abs(refv).max()) if refv.size else 0.0
    row_nnz = int(np.diff(A.indptr).max()) if A.rows else 0
    return float(8.0 * eps * max(1, row_nnz) * scale + 1e-12)


@dataclass
class VerifyResult:
    kernel: str
    matrix_class: str
    backend: str
    rows: int = 0
    nnz: int = 0
    max_abs_err: float = 0.0
    max_rel_err: float = 0.0
    tolerance: float = 0.0
    ok: bool = False
    inject_bug: bool = False
    message: str = ""
    config: Dict[str, Any] = field(default_factory=dict)

    def to_dict(self) -> Dict[str, Any]:
        return dict(self.__dict__)


def run_kernel(gen: "_codegen.B200Kernel", A: CSR, data, K: int = 8) -> np.ndarray:
    """Run the b200 kernel described by `gen` on device copies of A and `data`; returns
    the output on the host (fp64)."""
    import torch

    from . import device as D

    dt = torch.float64 if gen.config.dtype == "f64" else torch.float32
    dev = torch.device("cuda", torch.cuda.current_device())
    x, w, B, U, V, alpha, beta = data
    T = lambda a: torch.as_tensor(np.ascontiguousarray(a)).to(dev, dtype=dt)  # noqa: E731
    k = gen.kernel_name
    if k == "axpy":
        out = D.axpy(T(x), T(w), alpha, beta, sched=gen)
    else:
        Ad = D.DeviceCSR.from_host(A, dev, dt)
        if k == "spmv":
            out = D.spmv(Ad, T(x), y=torch.zeros(A.rows, dtype=dt, device=dev), sched=gen)
        elif k == "fused_spmv_axpy":
            out = D.fused_spmv_axpy(Ad, T(x), T(w), alpha, beta, z=torch.zeros(A.rows, dtype=dt, device=dev),
                                    sched=gen)
        elif k == "spmm":
            out = D.spmm(Ad, T(B), C=torch.zeros((A.rows, K), dtype=dt, device=dev), sched=gen)
        elif k == "sddmm":
            out = D.sddmm(Ad, T(U), T(V), out=torch.zeros(A.nnz, dtype=dt, device=dev), sched=gen)
        else:
            raise ValueError("unknown kernel %r" % k)
    torch.cuda.synchronize(dev)
    return out.double().cpu().numpy()


def run_launcher(kernel_name: str, A: CSR, data, K: int = 8, sched: "_lib.TgSched" = None) -> np.ndarray:
    """Call the reference-ABI ``launch_<kernel_name>`` of the library on device buffers
    (fp64), as tilegen/verify.py:414-451 does for a generated CUDA object."""
    import torch

    L = _lib.load()
    if sched is not None:
        _lib.set_schedule(sched)
    dev = torch.device("cuda", torch.cuda.current_device())
    x, w, B, U, V, alpha, beta = data
    T = lambda a: torch.as_tensor(np.ascontiguousarray(a, dtype=np.float64)).to(dev)  # noqa: E731
    M, N = A.shape
    nnz = A.nnz
    ip = torch.as_tensor(A.indptr).to(dev)
    ix = torch.as_tensor(A.indices).to(dev)
    dv = T(A.data)
    p = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    # every device buffer is bound to a name until the synchronous call returns
    if kernel_name == "spmv":
        dx = T(x)
        out = torch.zeros(M, dtype=torch.float64, device=dev)
        L.launch_spmv(p(ip), p(ix), p(dv), p(dx), p(out), M, N, nnz)
    elif kernel_name == "spmm":
        dB = T(B)
        out = torch.zeros((M, K), dtype=torch.float64, device=dev)
        L.launch_spmm(p(ip), p(ix), p(dv), p(dB), p(out), M, N, K, nnz)
    elif kernel_name == "sddmm":
        dU, dV = T(U), T(V)
        out = torch.zeros(nnz, dtype=torch.float64, device=dev)
        L.launch_sddmm(p(ip), p(ix), p(dv), p(dU), p(dV), p(out), M, N, K, nnz)
    elif kernel_name == "fused_spmv_axpy":
        dx, dw = T(x), T(w)
        out = torch.zeros(M, dtype=torch.float64, device=dev)
        L.launch_fused_spmv_axpy(p(ip), p(ix), p(dv), p(dx), p(dw), p(out), alpha, beta, M, N, nnz)
    elif kernel_name == "axpy":
        dx, dw = T(x), T(w)
        out = torch.zeros(M, dtype=torch.float64, device=dev)
        L.launch_axpy(p(dx), p(dw), p(out), alpha, beta, M)
    else:
        raise ValueError("unknown kernel %r" % kernel_name)
    status = L.tg_last_status()
    if status != _lib.TG_OK:
        raise _lib.TgError(status, "launch_%s" % kernel_name, _lib.last_error())
    return out.cpu().numpy()


def verify(kernel_name: str, config: "_codegen.Config", matrix, backend: str = "b200", workdir: str = None,
           K: int = 8, seed: int = 7, skip_passes: Sequence[str] = ()) -> VerifyResult:
    """Generate (descriptor), run and compare one kernel against SciPy float64."""
    if kernel_name not in KERNELS:
        raise ValueError("unknown kernel %r" % kernel_name)
    A, class_name = load_matrix(matrix)
    data = inputs_for(kernel_name, A, K, seed)
    refv = np.asarray(reference(kernel_name, A, data), dtype=np.float64).ravel()
    gen = _codegen.generate(kernel_name, config, backend, outdir=workdir, write=bool(workdir),
                            skip_passes=skip_passes)
    try:
        _, log = _codegen.compile_generated(gen, backend)
        out = run_kernel(gen, A, data, K).ravel()
    except _lib.TgError as exc:
        return VerifyResult(kernel_name, class_name, backend, A.rows, A.nnz, ok=False, inject_bug=config.inject_bug,
                            message="kernel error: %s" % exc, config=config.to_dict())
    diff = np.abs(out - refv)
    max_abs = float(diff.max()) if diff.size else 0.0
    denom = np.maximum(np.abs(refv), 1e-300)
    max_rel = float((diff / denom).max()) if diff.size else 0.0
    tol = tolerance(A, refv, config.dtype)
    return VerifyResult(kernel_name, class_name, backend, A.rows, A.nnz, max_abs, max_rel, tol,
                        bool(max_abs <= tol), config.inject_bug, log, config.to_dict())
