"""tg_spmv_f64_noalloc: the merge-split SpMV for callers that cannot allocate device
memory (a host that owns the whole GPU pool, or a path that cannot take cudaMalloc's
implicit synchronisation).  Its scratch is a fixed device array inside the library.

Checked through the C ABI against the allocating entry point tg_spmv_f64 (same split,
caller workspace) and against the CPU oracle, within the fp64 bar of the other parity
tests, on two calls in a row (the second call reuses the array the first one left
behind), then on a smaller and a larger matrix right after (left-over partition table
or split-row partials of an earlier call must not leak into the next), and on a matrix
without nonzeros.  This file is collected last so that a run stopping at the first
failure has run everything else.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from oracle import oracle as O
from tilegen_b200 import codegen as cg
from tilegen_b200 import device as D
from tilegen_b200 import lib
from tilegen_b200 import matrices as M
from tilegen_b200.verify import tolerance

pytestmark = pytest.mark.gpu


def _rel(out, ref):
    floor = 1e-3 * max(float(np.abs(ref).max()), 1e-300) if ref.size else 1.0
    return float((np.abs(out - ref) / np.maximum(np.abs(ref), floor)).max()) if ref.size else 0.0


def _noalloc(L, A, x, y, sched):
    desc = A.desc()
    return L.tg_spmv_f64_noalloc(ctypes.byref(desc), x.data_ptr(), y.data_ptr(),
                                 ctypes.byref(sched) if sched is not None else None,
                                 torch.cuda.current_stream().cuda_stream)


def _check_one(L, m, seed, sched, calls):
    A = D.DeviceCSR.from_host(m, "cuda")
    xh = np.random.default_rng(seed).uniform(-1, 1, m.cols)
    x = torch.as_tensor(xh).cuda()
    ref = D.spmv(A, x, sched=sched)  # tg_spmv_f64 with a caller workspace
    torch.cuda.synchronize()
    ref_h = ref.cpu().numpy()
    oracle = O.spmv(m, xh)
    tol = tolerance(m, oracle)
    for call in range(calls):
        y = torch.full((m.rows,), np.nan, dtype=torch.float64, device="cuda")
        st = _noalloc(L, A, x, y, sched)
        assert st == lib.TG_OK, lib.last_error()
        torch.cuda.synchronize()
        out = y.cpu().numpy()
        d_ref = float(np.abs(out - ref_h).max()) if m.rows else 0.0
        d_orc = float(np.abs(out - oracle).max()) if m.rows else 0.0
        assert d_ref <= tol, "%s call %d: max abs diff to tg_spmv_f64 %.3g > %.3g" % (m.name, call, d_ref, tol)
        assert d_orc <= tol, "%s call %d: max abs diff to the oracle %.3g > %.3g" % (m.name, call, d_orc, tol)
        assert _rel(out, oracle) <= 1e-9


def test_no_alloc_matches_allocating_entry_point_and_oracle_twice():
    assert torch.cuda.is_available()
    L = lib.load()
    sched = cg.generate("spmv", cg.Config(split="merge", block_size=256)).sched
    # power-law rows: many rows cross the merge chunks, so the split-row counters and
    # partials in the shared scratch are exercised
    _check_one(L, M.baseline_matrix("c3", scale=0.3), 21, sched, calls=2)


def test_no_alloc_smaller_then_larger_matrix_after_earlier_calls():
    L = lib.load()
    sched = cg.generate("spmv", cg.Config(split="merge", block_size=256)).sched
    _check_one(L, M.baseline_matrix("c3", scale=0.3), 21, sched, calls=1)
    _check_one(L, M.baseline_matrix("c3", scale=0.05), 22, sched, calls=1)  # fewer chunks than before
    _check_one(L, M.baseline_matrix("c3", scale=0.8), 23, sched, calls=1)   # more chunks than before
    _check_one(L, M.make_matrix("dense_rows"), 24, None, calls=1)           # NULL schedule


def test_no_alloc_without_nonzeros_writes_zeros():
    L = lib.load()
    dev = torch.device("cuda")
    A = D.DeviceCSR(torch.zeros(6, dtype=torch.int64, device=dev), torch.zeros(0, dtype=torch.int64, device=dev),
                    torch.zeros(0, dtype=torch.float64, device=dev), (5, 7))
    y = torch.full((5,), 7.0, dtype=torch.float64, device=dev)
    x = torch.ones(7, dtype=torch.float64, device=dev)
    assert _noalloc(L, A, x, y, None) == lib.TG_OK, lib.last_error()
    torch.cuda.synchronize()
    assert torch.all(y == 0)


def test_no_alloc_rejects_sizes_beyond_its_scratch():
    """The size check runs before any device access: a descriptor claiming 10^9
    nonzeros is refused with the limit in the message."""
    L = lib.load()
    big = lib.TgCsr(1000, 1000, 10 ** 9, 16, 16, 16)  # never dereferenced
    st = L.tg_spmv_f64_noalloc(ctypes.byref(big), 16, 16, None, None)
    assert st == lib.TG_EINVAL
    assert "scratch" in lib.last_error() and "nonzeros" in lib.last_error()
