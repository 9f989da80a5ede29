"""tg_spmv_f64_noalloc: the merge-split SpMV for callers that cannot allocate device
memory (a host that owns the whole GPU pool, or a path that cannot take cudaMalloc's
implicit synchronisation).  Its scratch is a fixed device array inside the library.

Checked through the C ABI against the allocating entry point tg_spmv_f64 (same split,
caller workspace), within the fp64 tolerance the other parity tests use, on two calls in
a row (the second call reuses the array the first one left behind).  This file is
collected last so that a run stopping at the first failure has run everything else.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from tilegen_b200 import codegen as cg
from tilegen_b200 import device as D
from tilegen_b200 import lib
from tilegen_b200 import matrices as M
from tilegen_b200.verify import tolerance

pytestmark = pytest.mark.gpu


def _matrix():
    # power-law rows: many rows cross the merge chunks, so the split-row counters and
    # partials in the shared scratch are exercised
    return M.baseline_matrix("c3", scale=0.3)


def test_no_alloc_matches_allocating_entry_point_twice():
    assert torch.cuda.is_available()
    L = lib.load()
    m = _matrix()
    A = D.DeviceCSR.from_host(m, "cuda")
    x = torch.as_tensor(np.random.default_rng(21).uniform(-1, 1, m.cols)).cuda()
    sched = cg.generate("spmv", cg.Config(split="merge", block_size=256)).sched
    ref = D.spmv(A, x, sched=sched)  # tg_spmv_f64 with a caller workspace
    torch.cuda.synchronize()
    ref_h = ref.cpu().numpy()
    tol = tolerance(m, ref_h)
    desc = A.desc()
    for call in range(2):
        y = torch.full((m.rows,), np.nan, dtype=torch.float64, device="cuda")
        st = L.tg_spmv_f64_noalloc(ctypes.byref(desc), x.data_ptr(), y.data_ptr(), ctypes.byref(sched),
                                   torch.cuda.current_stream().cuda_stream)
        assert st == lib.TG_OK, lib.last_error()
        torch.cuda.synchronize()
        d = float(np.abs(y.cpu().numpy() - ref_h).max())
        assert d <= tol, "call %d: max abs diff %.3g > %.3g" % (call, d, tol)


def test_no_alloc_rejects_sizes_beyond_its_scratch():
    """The size check runs before any device access: a descriptor claiming 10^9
    nonzeros is refused with the limit in the message."""
    L = lib.load()
    big = lib.TgCsr(1000, 1000, 10 ** 9, 16, 16, 16)  # never dereferenced
    st = L.tg_spmv_f64_noalloc(ctypes.byref(big), 16, 16, None, None)
    assert st == lib.TG_EINVAL
    assert "scratch" in lib.last_error() and "nonzeros" in lib.last_error()
