"""Device-side calls of the b200 kernels on torch tensors.

PyTorch provides the device memory and the stream; the arithmetic runs in
libtilegen_b200.so through its native C ABI (``tg_*``).  Every call is asynchronous on
the given (default: current) torch CUDA stream.  Workspace for the merge split is
allocated here, on the Python side, and cached per device (grow-only); calls that run
concurrently on different streams of one device must pass their own ``workspace``.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Dict, Optional, Tuple

import numpy as np
import torch

from . import lib as _lib
from .matrices import CSR

__all__ = ["DeviceCSR", "spmv", "fused_spmv_axpy", "spmm", "sddmm", "axpy", "workspace_for"]

_TORCH_OF = {"f64": torch.float64, "f32": torch.float32}


def _dev(device) -> torch.device:
    d = torch.device(device)
    if d.type != "cuda":
        raise ValueError("b200 kernels run on CUDA devices only (got %s)" % d)
    if d.index is None:
        d = torch.device("cuda", torch.cuda.current_device())
    return d


@dataclass
class DeviceCSR:
    """CSR operand resident on one GPU (int64 indptr/indices, fp64 or fp32 values)."""

    indptr: torch.Tensor
    indices: torch.Tensor
    data: torch.Tensor
    shape: Tuple[int, int]

    @property
    def rows(self) -> int:
        return int(self.shape[0])

    @property
    def cols(self) -> int:
        return int(self.shape[1])

    @property
    def nnz(self) -> int:
        return int(self.indices.numel())

    @property
    def device(self) -> torch.device:
        return self.indptr.device

    @classmethod
    def from_host(cls, m: CSR, device="cuda", dtype: torch.dtype = torch.float64,
                  non_blocking: bool = False) -> "DeviceCSR":
        d = _dev(device)
        ip = torch.as_tensor(np.ascontiguousarray(m.indptr, dtype=np.int64)).to(d, non_blocking=non_blocking)
        ix = torch.as_tensor(np.ascontiguousarray(m.indices, dtype=np.int64)).to(d, non_blocking=non_blocking)
        dv = torch.as_tensor(np.ascontiguousarray(m.data)).to(d, dtype=dtype, non_blocking=non_blocking)
        return cls(ip, ix, dv, (m.rows, m.cols))

    def desc(self) -> _lib.TgCsr:
        for t, name in ((self.indptr, "indptr"), (self.indices, "indices")):
            if t.dtype != torch.int64 or not t.is_contiguous():
                raise TypeError("%s must be a contiguous int64 tensor" % name)
        if not self.data.is_contiguous():
            raise TypeError("data must be contiguous")
        return _lib.TgCsr(self.rows, self.cols, self.nnz, self.indptr.data_ptr(),
                          self.indices.data_ptr() if self.nnz else 0, self.data.data_ptr() if self.nnz else 0)


_WS: Dict[int, torch.Tensor] = {}


def workspace_for(nbytes: int, device: torch.device) -> Tuple[int, int]:
    """(pointer, size) of the cached per-device workspace, grown to >= nbytes."""
    if nbytes <= 0:
        return 0, 0
    idx = _dev(device).index
    buf = _WS.get(idx)
    if buf is None or buf.numel() < nbytes:
        torch.cuda.synchronize(idx)  # the old buffer may still be in use by queued work
        buf = torch.empty(int(nbytes), dtype=torch.uint8, device=torch.device("cuda", idx))
        _WS[idx] = buf
    return buf.data_ptr(), buf.numel()


def _sched(sched) -> _lib.TgSched:
    if sched is None:
        return _lib.default_schedule()
    if isinstance(sched, _lib.TgSched):
        return sched
    if hasattr(sched, "sched"):  # a codegen.B200Kernel
        return sched.sched
    raise TypeError("sched must be a TgSched or a B200Kernel")


def _stream_ptr(stream: Optional[torch.cuda.Stream], device: torch.device) -> int:
    s = stream if stream is not None else torch.cuda.current_stream(device)
    return int(s.cuda_stream)


def _check_vec(t: torch.Tensor, n: int, dtype: torch.dtype, device: torch.device, name: str) -> None:
    if t.device != device or t.dtype != dtype or not t.is_contiguous() or t.numel() != n:
        raise ValueError("%s must be a contiguous %s tensor of %d elements on %s (got %s %s %s)"
                         % (name, dtype, n, device, tuple(t.shape), t.dtype, t.device))


def _ws(nbytes: int, device, workspace) -> Tuple[int, int]:
    if workspace is not None:
        if workspace.numel() * workspace.element_size() < nbytes:
            raise ValueError("workspace too small: need %d bytes" % nbytes)
        return workspace.data_ptr(), workspace.numel() * workspace.element_size()
    return workspace_for(nbytes, device)


def spmv(A: DeviceCSR, x: torch.Tensor, y: Optional[torch.Tensor] = None, sched=None,
         stream: Optional[torch.cuda.Stream] = None, workspace: Optional[torch.Tensor] = None) -> torch.Tensor:
    """y = A x (fp64, or fp32 with fp32 accumulation when A.data is float32)."""
    L = _lib.load()
    dt = A.data.dtype
    dev = A.device
    s = _sched(sched)
    _check_vec(x, A.cols, dt, dev, "x")
    if y is None:
        y = torch.empty(A.rows, dtype=dt, device=dev)
    _check_vec(y, A.rows, dt, dev, "y")
    nbytes = L.tg_spmv_workspace_bytes(A.rows, A.nnz, ctypes.byref(s))
    wp, wn = _ws(nbytes, dev, workspace)
    fn = L.tg_spmv_f64 if dt == torch.float64 else L.tg_spmv_f32
    desc = A.desc()
    _lib.check(fn(ctypes.byref(desc), x.data_ptr(), y.data_ptr(), ctypes.byref(s), wp, wn, _stream_ptr(stream, dev)),
               "tg_spmv")
    return y


def fused_spmv_axpy(A: DeviceCSR, x: torch.Tensor, w: torch.Tensor, alpha: float, beta: float,
                    z: Optional[torch.Tensor] = None, sched=None, stream=None,
                    workspace: Optional[torch.Tensor] = None) -> torch.Tensor:
    """z = alpha * (A x) + beta * w (fp64, or fp32 with fp32 accumulation when A.data is
    float32)."""
    L = _lib.load()
    dev = A.device
    dt = A.data.dtype
    s = _sched(sched)
    _check_vec(x, A.cols, dt, dev, "x")
    _check_vec(w, A.rows, dt, dev, "w")
    if z is None:
        z = torch.empty(A.rows, dtype=dt, device=dev)
    _check_vec(z, A.rows, dt, dev, "z")
    nbytes = L.tg_spmv_workspace_bytes(A.rows, A.nnz, ctypes.byref(s))
    wp, wn = _ws(nbytes, dev, workspace)
    desc = A.desc()
    fn = L.tg_fused_spmv_axpy_f64 if dt == torch.float64 else L.tg_fused_spmv_axpy_f32
    _lib.check(fn(ctypes.byref(desc), x.data_ptr(), w.data_ptr(), z.data_ptr(), float(alpha), float(beta),
                  ctypes.byref(s), wp, wn, _stream_ptr(stream, dev)), "tg_fused_spmv_axpy")
    return z


def spmm(A: DeviceCSR, B: torch.Tensor, C: Optional[torch.Tensor] = None, sched=None, stream=None,
         workspace: Optional[torch.Tensor] = None) -> torch.Tensor:
    """C = A B with B (cols x K) and C (rows x K) row-major; C is overwritten."""
    L = _lib.load()
    dt = A.data.dtype
    dev = A.device
    s = _sched(sched)
    if B.dim() != 2 or B.shape[0] != A.cols:
        raise ValueError("B must be (cols x K)")
    K = int(B.shape[1])
    _check_vec(B.reshape(-1), A.cols * K, dt, dev, "B")
    if C is None:
        C = torch.empty((A.rows, K), dtype=dt, device=dev)
    _check_vec(C.reshape(-1), A.rows * K, dt, dev, "C")
    nbytes = L.tg_spmm_workspace_bytes(A.rows, A.nnz, K, ctypes.byref(s))
    wp, wn = _ws(nbytes, dev, workspace)
    fn = L.tg_spmm_f64 if dt == torch.float64 else L.tg_spmm_f32
    desc = A.desc()
    _lib.check(fn(ctypes.byref(desc), B.data_ptr(), C.data_ptr(), K, ctypes.byref(s), wp, wn,
                  _stream_ptr(stream, dev)), "tg_spmm")
    return C


def sddmm(A: DeviceCSR, U: torch.Tensor, V: torch.Tensor, out: Optional[torch.Tensor] = None, sched=None,
          stream=None, workspace: Optional[torch.Tensor] = None) -> torch.Tensor:
    """out[p] = A.data[p] * dot(U[i], V[j]) on A's pattern (values in A's order)."""
    L = _lib.load()
    dt = A.data.dtype
    dev = A.device
    s = _sched(sched)
    if U.dim() != 2 or V.dim() != 2 or U.shape[0] != A.rows or V.shape[0] != A.cols or U.shape[1] != V.shape[1]:
        raise ValueError("U must be (rows x K) and V (cols x K)")
    K = int(U.shape[1])
    _check_vec(U.reshape(-1), A.rows * K, dt, dev, "U")
    _check_vec(V.reshape(-1), A.cols * K, dt, dev, "V")
    if out is None:
        out = torch.empty(A.nnz, dtype=dt, device=dev)
    _check_vec(out, A.nnz, dt, dev, "out")
    nbytes = L.tg_sddmm_workspace_bytes(A.rows, A.nnz, K, ctypes.byref(s))
    wp, wn = _ws(nbytes, dev, workspace)
    fn = L.tg_sddmm_f64 if dt == torch.float64 else L.tg_sddmm_f32
    desc = A.desc()
    _lib.check(fn(ctypes.byref(desc), U.data_ptr(), V.data_ptr(), out.data_ptr(), K, ctypes.byref(s), wp, wn,
                  _stream_ptr(stream, dev)), "tg_sddmm")
    return out


def axpy(x: torch.Tensor, w: torch.Tensor, alpha: float, beta: float, z: Optional[torch.Tensor] = None,
         sched=None, stream=None) -> torch.Tensor:
    """z = alpha x + beta w (fp64, or fp32 when x is float32)."""
    L = _lib.load()
    dev = x.device
    dt = x.dtype
    if dt not in (torch.float64, torch.float32):
        raise ValueError("axpy operands must be float64 or float32 (got %s)" % dt)
    s = _sched(sched)
    n = x.numel()
    _check_vec(x, n, dt, dev, "x")
    _check_vec(w, n, dt, dev, "w")
    if z is None:
        z = torch.empty(n, dtype=dt, device=dev)
    _check_vec(z, n, dt, dev, "z")
    fn = L.tg_axpy_f64 if dt == torch.float64 else L.tg_axpy_f32
    _lib.check(fn(x.data_ptr(), w.data_ptr(), z.data_ptr(), float(alpha), float(beta), n, ctypes.byref(s),
                  _stream_ptr(stream, dev)), "tg_axpy")
    return z
