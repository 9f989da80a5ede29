"""Row-sharded power iteration x <- A x / ||A x|| on one GPU per process.

The multi-GPU mode of the hot path (no counterpart in the reference, whose kernels run on
one device).  Rows of A are split into P contiguous, nnz-balanced shards, one per rank;
x is replicated.  The iterate lives in a padded vector of P * stride doubles (shard r at
r * stride, its sum of squares in the shard's last element, the slot -- see
include/tilegen_b200.h), and the column indices of each shard are renumbered once to that
layout, so the all-gather of the output shards *is* the next iterate: no compaction, no
separate norm all-reduce (every rank sums the P slots it received), and the 1/||y|| scale
is applied inside the next step's kernel.

``PowerIteration`` drives one rank.  Its exchange step is pluggable: by default an
in-place ``torch.distributed.all_gather_into_tensor`` (NCCL over NVLink/NVSwitch), no
exchange at P = 1.  The local step is the C ABI's ``tg_power_step_f64``; tests on CPU
substitute a host implementation of the same contract.
"""

from __future__ import annotations

import ctypes
from typing import Callable, List, Optional, Sequence, Tuple

import numpy as np

__all__ = ["nnz_balanced_bounds", "uniform_bounds", "padded_stride", "renumber_columns", "PowerIteration"]


def nnz_balanced_bounds(row_nnz: np.ndarray, parts: int) -> np.ndarray:
    """Row boundaries b[0..parts] so rank r owns rows [b[r], b[r+1]) with about nnz/parts
    nonzeros each: b[r] is the first row whose nnz prefix reaches r * nnz / parts."""
    if parts < 1:
        raise ValueError("parts must be >= 1")
    csum = np.concatenate([[0], np.cumsum(np.asarray(row_nnz, dtype=np.int64))])
    total = int(csum[-1])
    rows = csum.size - 1
    b = np.empty(parts + 1, dtype=np.int64)
    b[0], b[parts] = 0, rows
    for r in range(1, parts):
        b[r] = int(np.searchsorted(csum, (r * total) // parts, side="left"))
    return np.maximum.accumulate(b)


def uniform_bounds(rows: int, parts: int) -> np.ndarray:
    """Equal row blocks (the nnz-balanced split of a constant-row-length matrix)."""
    return np.array([(r * rows) // parts for r in range(parts + 1)], dtype=np.int64)


def padded_stride(bounds: np.ndarray, align: int = 32) -> int:
    """Shard stride: the largest shard plus one slot, rounded up to `align` doubles."""
    longest = int(np.max(np.diff(bounds))) if bounds.size > 1 else 0
    return ((longest + 1 + align - 1) // align) * align


def renumber_columns(indices, bounds, stride: int, index32: bool = False):
    """j -> owner(j) * stride + (j - bounds[owner(j)]).  CUDA tensors go through the
    library's kernel (tg_renumber_columns, or tg_renumber_columns_i32 with ``index32``:
    int32 output, which the power steps read with TG_FLAG_INDEX32), on the current
    stream; numpy arrays and CPU tensors are renumbered on the host (the gloo tests)."""
    try:
        import torch

        if isinstance(indices, torch.Tensor):
            if indices.is_cuda:
                from . import lib as _lib

                L = _lib.load()
                idx = indices.contiguous().to(torch.int64)
                out = torch.empty(idx.numel(), dtype=torch.int32 if index32 else torch.int64, device=idx.device)
                fn = L.tg_renumber_columns_i32 if index32 else L.tg_renumber_columns
                b = np.ascontiguousarray(bounds, dtype=np.int64)
                with torch.cuda.device(idx.device):
                    st = torch.cuda.current_stream(idx.device).cuda_stream
                    _lib.check(fn(idx.data_ptr(), out.data_ptr(), idx.numel(), b.ctypes.data, b.size - 1, int(stride),
                                  st), "tg_renumber_columns")
                return out
            return torch.from_numpy(renumber_columns(indices.numpy(), bounds, stride))
    except ImportError:  # pragma: no cover
        pass
    b = np.asarray(bounds, dtype=np.int64)
    owner = np.searchsorted(b, indices, side="right") - 1
    return owner * stride + (indices - b[owner])


class _Exchange:
    """State of the fused exchange: this rank's iterate buffers, the peers' mapped
    buffers and flag arrays (as pointer arrays for the C ABI), and the epoch counter,
    which keeps increasing for as long as the flag arrays are in use."""

    def __init__(self):
        self.y_ptrs = None
        self.flag_ptrs = None
        self.flags_local = None
        self.keep = None
        self.x = None
        self.epoch = 0
        self.owned = []
        self.opened = []
        self.group = None


class _PeerPtr:
    """A device address mapped from another rank (only its data_ptr is used)."""

    def __init__(self, ptr: int):
        self.ptr = int(ptr)

    def data_ptr(self) -> int:
        return self.ptr


class _CudaArray:
    def __init__(self, ptr: int, n: int, typestr: str):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": typestr, "data": (int(ptr), False),
                                         "version": 3, "strides": None}


def _device_view(ptr: int, n: int, dtype, device):
    """A torch tensor over n elements of device memory at ptr (no copy, not owning)."""
    import torch

    typestr = {torch.float64: "<f8", torch.int64: "<i8"}[dtype]
    with torch.cuda.device(device):
        return torch.as_tensor(_CudaArray(ptr, n, typestr), device=device)


class PowerIteration:
    """One rank of the sharded power iteration.

    Parameters: the rank's CSR shard on its device as torch tensors (indptr rebased to 0,
    ORIGINAL global column indices), the global row bounds, this rank, and optionally a
    custom ``step`` (signature ``step(x_full, y_shard)``), ``norm2`` (``norm2(shard)``),
    ``finalize`` (``finalize(x_full, x_out, lam_out)``) and ``exchange``
    (``exchange(x_full)``, all-gathers the shards in place).  The custom hooks exist for
    host-side tests of the sharding logic; the defaults are the GPU kernels.

    ``index32`` keeps the renumbered column indices as int32 (the GPU steps, rowwise
    split, padded layout below 2^31 entries), so every step streams 12 bytes per nonzero
    instead of 16; the matrix is renumbered once, here, and read by every step.  The
    default (None) turns it on with 16-byte index loads (vector_width 4), the schedule
    where it measured faster on the 8M-row C4 matrix (1.193 ms per step at TPR4 U1 V4,
    against 1.234 ms for the best int64 schedule, TPR4 U2 V2); with pairs of indices
    (vector_width 2) it measured slower (1.301 ms) and stays off.
    """

    def __init__(self, indptr, indices, data, bounds: Sequence[int], rank: int, sched=None,
                 step: Optional[Callable] = None, norm2: Optional[Callable] = None,
                 finalize: Optional[Callable] = None, exchange: Optional[Callable] = None,
                 renumber: bool = True, index32: Optional[bool] = None):
        import torch

        self.torch = torch
        self.bounds = np.asarray(bounds, dtype=np.int64)
        self.parts = int(self.bounds.size - 1)
        self.rank = int(rank)
        self.rows = int(self.bounds[rank + 1] - self.bounds[rank])
        self.cols = int(self.bounds[-1])
        self.stride = padded_stride(self.bounds)
        self.device = indptr.device
        if int(indptr.numel()) != self.rows + 1:
            raise ValueError("indptr has %d entries for a %d-row shard" % (indptr.numel(), self.rows))
        self.indptr = indptr
        gpu = step is None and norm2 is None and finalize is None and getattr(indices, "is_cuda", False)
        fits = gpu and renumber and self.parts * self.stride < 2 ** 31
        if index32 is None:
            s0 = sched if sched is not None else None
            split = getattr(s0, "split", 0) if s0 is not None else 0
            vec = getattr(s0, "vector_width", 4) if s0 is not None else 4
            index32 = fits and split == 0 and vec == 4
        if index32 and not fits:
            raise ValueError("index32 needs the GPU steps, renumber=True and a padded layout below 2^31")
        self.index32 = bool(index32)
        self.indices = (renumber_columns(indices, self.bounds, self.stride, self.index32) if renumber else indices)
        self.data = data
        self.nnz = int(indices.numel())
        n = self.parts * self.stride
        self.x = [torch.zeros(n, dtype=torch.float64, device=self.device) for _ in range(2)]
        self.cur = 0
        self.sched = sched
        self._step = step or self._gpu_step
        self._norm2 = norm2 or self._gpu_norm2
        self._finalize = finalize or self._gpu_finalize
        self._exchange = exchange or (self._nccl_exchange if self.parts > 1 else (lambda x: None))
        self.kernel_launches = 0
        self.p2p = False
        # exchange over peer memory: "store" (tg_power_step_p2p_f64: the computing warps
        # store every finished tile into every rank) or "ce" (tg_power_step_ce_f64: the
        # step in row chunks, each chunk copied to every peer by the copy engines while
        # the next one computes)
        self.p2p_mode = "store"
        self.ce_chunks = 4  # "ce": row chunks whose copies overlap the next chunk's compute
        self._ex = None
        if step is None or norm2 is None or finalize is None:
            from . import lib as _lib

            self._lib = _lib
            L = _lib.load()
            self._sched_c = sched if sched is not None else self._default_sched()
            if self.index32:
                self._sched_c = self._lib.TgSched(*[getattr(self._sched_c, f) for f, _ in self._sched_c._fields_])
                self._sched_c.flags |= self._lib.TG_FLAG_INDEX32
            self.ws = torch.zeros(int(L.tg_power_workspace_bytes(self.nnz, ctypes.byref(self._sched_c))),
                                  dtype=torch.uint8, device=self.device)
            self._desc = _lib.TgCsr(self.rows, n, self.nnz, self.indptr.data_ptr(), self.indices.data_ptr(),
                                    self.data.data_ptr())
            self._planned = False

    # -- shard views -------------------------------------------------------------------
    def shard(self, buf) -> "object":
        o = self.rank * self.stride
        return buf[o:o + self.stride]

    # -- GPU implementations -----------------------------------------------------------
    def _default_sched(self):
        s = self._lib.default_schedule()
        # the fastest power-step schedule measured on the 8M-row uniform matrix (with int32
        # renumbered indices, chosen by default for it)
        s.threads_per_row, s.unroll, s.vector_width, s.block_size, s.tile = 4, 1, 4, 256, 32
        s.split = self._lib.TG_SPLIT_ROWWISE
        return s

    def _stream(self) -> int:
        return int(self.torch.cuda.current_stream(self.device).cuda_stream)

    def _gpu_step(self, x_full, y_shard) -> None:
        L = self._lib.load()
        s = self._sched_c
        if self._planned:  # the partition of this matrix is already in the workspace
            s = self._lib.TgSched(*[getattr(s, f) for f, _ in s._fields_])
            s.flags |= self._lib.TG_FLAG_REUSE_PLAN
        self._lib.check(L.tg_power_step_f64(ctypes.byref(self._desc), x_full.data_ptr(), self.parts, self.stride,
                                            y_shard.data_ptr(), ctypes.byref(s), self.ws.data_ptr(),
                                            self.ws.numel(), self._stream()), "tg_power_step_f64")
        self.kernel_launches += 1 if self._planned or self._sched_c.split != self._lib.TG_SPLIT_STREAM else 3
        self._planned = True

    def _gpu_norm2(self, shard) -> None:
        L = self._lib.load()
        self._lib.check(L.tg_shard_norm2_f64(shard.data_ptr(), self.rows, self.stride, self.ws.data_ptr(),
                                             self.ws.numel(), self._stream()), "tg_shard_norm2_f64")
        self.kernel_launches += 1

    def _nccl_exchange(self, x_full) -> None:
        import torch.distributed as dist

        dist.all_gather_into_tensor(x_full, self.shard(x_full))

    # -- fused exchange over peer memory ------------------------------------------------
    def p2p_setup(self, peer_x, peer_flags) -> None:
        """Switch iterate() to the fused step (tg_power_step_p2p_f64).  peer_x[q] is the
        pair (x[0], x[1]) of rank q and peer_flags[q] its flag array (int64, zeroed),
        all accessible from this device (local tensors, or peer memory mapped by CUDA
        IPC); index self.rank must be this object's own x and flags."""
        if len(peer_x) != self.parts or len(peer_flags) != self.parts:
            raise ValueError("need one buffer pair and one flag array per rank")
        P = ctypes.c_void_p * 8
        ex = _Exchange()
        ex.y_ptrs = [P(*([int(px[b].data_ptr()) for px in peer_x] + [0] * (8 - self.parts))) for b in (0, 1)]
        ex.flag_ptrs = P(*([int(f.data_ptr()) for f in peer_flags] + [0] * (8 - self.parts)))
        ex.flags_local = peer_flags[self.rank]
        ex.keep = (peer_x, peer_flags)
        ex.x = [peer_x[self.rank][0], peer_x[self.rank][1]]
        self.p2p_attach(ex)

    def p2p_attach(self, ex: "_Exchange") -> None:
        """Use an existing exchange (buffers, peer mappings, flags and epoch counter),
        e.g. the one of another PowerIteration over a matrix with the same row bounds:
        the mappings do not depend on the matrix."""
        self._ex = ex
        self.x = ex.x
        self.p2p = True

    def p2p_connect(self, group=None) -> None:
        """Allocate x[0], x[1] and a zeroed flag array as peer-shareable buffers, exchange
        their CUDA IPC handles with every rank of the process group, map the peers'
        buffers into this device's context, then p2p_setup.  close() releases them."""
        import torch.distributed as dist

        torch = self.torch
        L = self._lib.load()
        n = self.parts * self.stride
        self._owned = []
        mine = []
        for nbytes in (8 * n, 8 * n, 8 * self.parts):
            p = ctypes.c_void_p()
            self._lib.check(L.tg_peer_buffer_alloc(nbytes, ctypes.byref(p)), "tg_peer_buffer_alloc")
            self._owned.append(p.value)
            h = ctypes.create_string_buffer(64)
            self._lib.check(L.tg_ipc_get_handle(p.value, h), "tg_ipc_get_handle")
            mine.append(h.raw)
        xa = _device_view(self._owned[0], n, torch.float64, self.device)
        xb = _device_view(self._owned[1], n, torch.float64, self.device)
        fl = _device_view(self._owned[2], self.parts, torch.int64, self.device)
        xa.copy_(self.x[0])
        xb.copy_(self.x[1])
        allh = [None] * self.parts
        dist.all_gather_object(allh, mine, group=group)
        self._opened = []
        peer_x, peer_flags = [], []
        for q, hs in enumerate(allh):
            if q == self.rank:
                peer_x.append((xa, xb))
                peer_flags.append(fl)
                continue
            ptrs = []
            for h in hs:
                p = ctypes.c_void_p()
                self._lib.check(L.tg_ipc_open(h, ctypes.byref(p)), "tg_ipc_open")
                self._opened.append(p.value)
                ptrs.append(p.value)
            peer_x.append((_PeerPtr(ptrs[0]), _PeerPtr(ptrs[1])))
            peer_flags.append(_PeerPtr(ptrs[2]))
        self.p2p_setup(peer_x, peer_flags)
        self._ex.owned, self._ex.opened, self._ex.group = self._owned, self._opened, group
        dist.barrier(group=group)

    def close(self) -> None:
        """Unmap the peers' buffers, then (after every rank did) free this rank's."""
        ex = getattr(self, "_ex", None)
        if ex is None or not ex.owned:
            return
        import torch.distributed as dist

        self.torch.cuda.synchronize(self.device)
        L = self._lib.load()
        for p in ex.opened:
            L.tg_ipc_close(p)
        ex.opened = []
        dist.barrier(group=ex.group)
        self.x = [self.x[0].clone(), self.x[1].clone()]
        ex.keep = None
        for p in ex.owned:
            L.tg_peer_buffer_free(p)
        ex.owned = []
        self.p2p = False

    def p2p_step(self, src_index: int) -> None:
        """One exchanged step: read self.x[src_index], and deliver this rank's shard of the
        result into every rank's other buffer (fused stores, or copies with
        ``p2p_mode == "ce"``)."""
        if self.p2p_mode == "ce":
            self._ce_step(src_index)
            return
        L = self._lib.load()
        ex = self._ex
        ex.epoch += 1
        self._lib.check(L.tg_power_step_p2p_f64(ctypes.byref(self._desc), self.x[src_index].data_ptr(), self.parts,
                                                self.rank, self.stride, ex.y_ptrs[1 - src_index], ex.flag_ptrs,
                                                ex.epoch, ctypes.byref(self._sched_c), self.ws.data_ptr(),
                                                self.ws.numel(), self._stream()), "tg_power_step_p2p_f64")
        self.kernel_launches += 1

    def _ce_step(self, src_index: int) -> None:
        L = self._lib.load()
        ex = self._ex
        ex.epoch += 1
        self._lib.check(L.tg_power_step_ce_f64(ctypes.byref(self._desc), self.x[src_index].data_ptr(), self.parts,
                                               self.rank, self.stride, ex.y_ptrs[1 - src_index], ex.flag_ptrs,
                                               ex.epoch, self.ce_chunks, ctypes.byref(self._sched_c),
                                               self.ws.data_ptr(), self.ws.numel(), self._stream()),
                        "tg_power_step_ce_f64")
        self.kernel_launches += self.ce_chunks + 2 + (1 if ex.epoch > 1 else 0)

    def p2p_wait(self) -> None:
        L = self._lib.load()
        self._lib.check(L.tg_p2p_wait(self._ex.flags_local.data_ptr(), self.parts, self._ex.epoch,
                                      self.ws.data_ptr(), self.ws.numel(), self._stream()), "tg_p2p_wait")
        self.kernel_launches += 1

    @property
    def exchange_state(self) -> "_Exchange":
        return self._ex

    def error_word(self) -> int:
        """The workspace's error word (synchronises the stream): 16 = a bounded wait for
        the peers ran out.  While it is set, fused steps and waits return at once."""
        L = self._lib.load()
        v = ctypes.c_uint32(0)
        self._lib.check(L.tg_power_error(self.ws.data_ptr(), ctypes.byref(v), self._stream()), "tg_power_error")
        return int(v.value)

    def clear_error(self) -> None:
        """Clear the error word.  A restart after a failed exchange also needs every
        rank's flag array zeroed and the epoch counter reset (reset_exchange)."""
        L = self._lib.load()
        self._lib.check(L.tg_power_clear_error(self.ws.data_ptr(), self._stream()), "tg_power_clear_error")

    def reset_exchange(self) -> None:
        """Zero this rank's flag array, restart the epoch count at 0 and clear the error
        word: the local half of a restart, which every rank must do (with its kernels
        finished) before any rank steps again."""
        self._ex.flags_local.zero_()
        self._ex.epoch = 0
        self.clear_error()

    # -- iteration ---------------------------------------------------------------------
    def set_x0(self, x0_local) -> None:
        """Start from x0 (this rank's rows); any scale (the first step normalises)."""
        xs = self.shard(self.x[0])
        xs.zero_()
        xs[:self.rows].copy_(x0_local)
        self._norm2(xs)
        self._exchange(self.x[0])
        self.cur = 0

    def iterate(self, iters: int, on_step: Optional[Callable[[int], None]] = None) -> None:
        for k in range(iters):
            src, dst = self.x[self.cur], self.x[1 - self.cur]
            if on_step:
                on_step(2 * k)
            if self.p2p:
                self.p2p_step(self.cur)
            else:
                self._step(src, self.shard(dst))
            if on_step:
                on_step(2 * k + 1)
            if not self.p2p:
                self._exchange(dst)
            self.cur = 1 - self.cur
        if self.p2p and iters > 0:
            self.p2p_wait()

    def _gpu_finalize(self, x_full, x_out, lam_out) -> None:
        L = self._lib.load()
        self._lib.check(L.tg_power_finalize_f64(x_full.data_ptr(), self.parts, self.stride, self.rank, self.rows,
                                                x_out.data_ptr(), lam_out.data_ptr(), self._stream()),
                        "tg_power_finalize_f64")
        self.kernel_launches += 1

    def result(self, x_out=None, lam_out=None) -> Tuple[object, object]:
        """(this rank's rows of the normalised iterate, ||A x_prev||) as tensors."""
        torch = self.torch
        if x_out is None:
            x_out = torch.empty(self.rows, dtype=torch.float64, device=self.device)
        if lam_out is None:
            lam_out = torch.empty(1, dtype=torch.float64, device=self.device)
        self._finalize(self.x[self.cur], x_out, lam_out)
        return x_out, lam_out
