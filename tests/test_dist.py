"""tg_dist_*: one process driving several GPUs (row shards, fused power-iteration exchange
over peer memory, SpMM / SDDMM without communication), against the oracle."""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

from oracle import oracle as O
from tilegen_b200 import lib
from tilegen_b200 import matrices as M


def _host_csr(m, data):
    return lib.TgCsr(m.rows, m.cols, m.nnz, m.indptr.ctypes.data, m.indices.ctypes.data, data.ctypes.data)


def _init(devices):
    L = lib.load()
    arr = (ctypes.c_int32 * len(devices))(*devices)
    h = ctypes.c_void_p()
    lib.check(L.tg_dist_init(len(devices), arr, ctypes.byref(h)), "tg_dist_init")
    return L, h


def rel(a, b):
    return float(np.abs(np.asarray(a, np.float64) - b).max() / max(np.abs(b).max(), 1e-300))


def test_dist_init_rejects_bad_arguments():
    L = lib.load()
    h = ctypes.c_void_p()
    assert L.tg_dist_init(0, (ctypes.c_int32 * 1)(0), ctypes.byref(h)) == lib.TG_EINVAL
    assert L.tg_dist_init(9, (ctypes.c_int32 * 9)(*range(9)), ctypes.byref(h)) == lib.TG_EINVAL
    assert L.tg_dist_init(2, (ctypes.c_int32 * 2)(0, 0), ctypes.byref(h)) == lib.TG_EINVAL
    assert "twice" in lib.last_error()
    assert L.tg_dist_init(1, (ctypes.c_int32 * 1)(0), None) == lib.TG_EINVAL
    assert L.tg_dist_finalize(None) == lib.TG_OK
    m = M.edge_matrix()
    A = _host_csr(m, m.data)
    lam = ctypes.c_double()
    assert L.tg_dist_spmv_power(None, ctypes.byref(A), None, 1, None, None, ctypes.byref(lam), 0.0) == lib.TG_EINVAL
    assert L.tg_dist_spmm_f32(None, ctypes.byref(A), None, 8, None, None, 0.0) == lib.TG_EINVAL
    assert L.tg_dist_sddmm_f32(None, ctypes.byref(A), None, None, 8, None, None, 0.0) == lib.TG_EINVAL


def _devices(n):
    import torch

    if torch.cuda.device_count() < n:
        pytest.skip("needs %d GPUs" % n)
    return list(range(n))


@pytest.mark.gpu
@pytest.mark.parametrize("n", [1, 2])
def test_dist_power_iteration_matches_oracle(n):
    L, h = _init(_devices(n))
    try:
        rows = 200_000
        A = M.c4_rows(0, rows, n=rows, per_row=32, seed=4)
        x0 = np.random.default_rng(1).uniform(-1, 1, rows)
        x = np.empty(rows)
        lam = ctypes.c_double()
        s = lib.default_schedule()
        s.threads_per_row, s.unroll, s.vector_width, s.block_size = 4, 2, 2, 256
        lib.check(L.tg_dist_spmv_power(h, ctypes.byref(_host_csr(A, A.data)), x0.ctypes.data, 20, ctypes.byref(s),
                                       x.ctypes.data, ctypes.byref(lam), 60.0), "tg_dist_spmv_power")
        xr, nr = O.power_iteration(A, x0, 20)
        assert rel(x, xr) <= 1e-9
        assert abs(lam.value - nr) <= 1e-9 * nr
    finally:
        assert L.tg_dist_finalize(h) == lib.TG_OK


@pytest.mark.gpu
@pytest.mark.parametrize("n", [1, 2])
def test_dist_spmm_sddmm_match_oracle(n):
    L, h = _init(_devices(n))
    try:
        m = M.baseline_matrix("c5", scale=0.05)
        d32 = m.data.astype(np.float32)
        m64 = M.CSR(m.indptr, m.indices, d32.astype(np.float64), m.shape, m.name)
        rng = np.random.default_rng(9)
        B = rng.uniform(-1, 1, (m.cols, 128)).astype(np.float32)
        U = rng.uniform(-1, 1, (m.rows, 64)).astype(np.float32)
        V = rng.uniform(-1, 1, (m.cols, 64)).astype(np.float32)
        C = np.empty((m.rows, 128), np.float32)
        out = np.empty(m.nnz, np.float32)
        s = lib.default_schedule()
        s.threads_per_row, s.unroll, s.vector_width, s.block_size, s.split = 32, 4, 4, 128, lib.TG_SPLIT_MERGE
        A = _host_csr(m, d32)
        lib.check(L.tg_dist_spmm_f32(h, ctypes.byref(A), B.ctypes.data, 128, C.ctypes.data, ctypes.byref(s), 60.0),
                  "tg_dist_spmm_f32")
        assert rel(C, O.spmm(m64, B.astype(np.float64))) <= 1e-4
        lib.check(L.tg_dist_sddmm_f32(h, ctypes.byref(A), U.ctypes.data, V.ctypes.data, 64, out.ctypes.data,
                                      ctypes.byref(s), 60.0), "tg_dist_sddmm_f32")
        assert rel(out, O.sddmm(m64, U.astype(np.float64), V.astype(np.float64))) <= 1e-4
    finally:
        assert L.tg_dist_finalize(h) == lib.TG_OK


@pytest.mark.gpu
def test_dist_host_deadline_then_context_still_usable():
    L, h = _init(_devices(1))
    try:
        rows = 400_000
        A = M.c4_rows(0, rows, n=rows, per_row=32, seed=4)
        x0 = np.ones(rows)
        x = np.empty(rows)
        lam = ctypes.c_double()
        # a deadline far shorter than 100 iterations on 12.8M nonzeros
        st = L.tg_dist_spmv_power(h, ctypes.byref(_host_csr(A, A.data)), x0.ctypes.data, 100, None, x.ctypes.data,
                                  ctypes.byref(lam), 1e-7)
        assert st == lib.TG_ETIMEDOUT and "did not finish" in lib.last_error()
        lib.check(L.tg_dist_spmv_power(h, ctypes.byref(_host_csr(A, A.data)), x0.ctypes.data, 3, None, x.ctypes.data,
                                       ctypes.byref(lam), 60.0), "tg_dist_spmv_power")
        xr, nr = O.power_iteration(A, x0, 3)
        assert rel(x, xr) <= 1e-9
    finally:
        assert L.tg_dist_finalize(h) == lib.TG_OK
