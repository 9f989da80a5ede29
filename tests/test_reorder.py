"""Column-locality reordering (tilegen_b200.reorder, tg_rcm_order): host logic on the CPU;
the permuted kernels on the GPU."""

from __future__ import annotations

import numpy as np
import pytest

from oracle import oracle as O
from tilegen_b200 import lib
from tilegen_b200 import matrices as M
from tilegen_b200 import reorder as R


def _band(n=5000, half=3, seed=1):
    rng = np.random.default_rng(seed)
    rows, cols = [], []
    for i in range(n):
        for j in range(max(0, i - half), min(n, i + half + 1)):
            rows.append(i)
            cols.append(j)
    rows, cols = np.array(rows), np.array(cols)
    indptr = np.zeros(n + 1, np.int64)
    np.add.at(indptr, rows + 1, 1)
    indptr = np.cumsum(indptr)
    return M.CSR(indptr, cols.astype(np.int64), rng.uniform(-1, 1, cols.size), (n, n), "band")


def test_rcm_is_a_permutation_and_recovers_a_scrambled_band():
    A = _band()
    S = R.scrambled(A, seed=3)
    assert R.bandwidth(S) > 1000
    perm = R.rcm_order(S)
    assert np.array_equal(np.sort(perm), np.arange(S.rows))
    B = R.permute(S, perm)
    assert R.bandwidth(B) <= 2 * R.bandwidth(A)


def test_permuted_spmv_and_spmm_are_the_permuted_results():
    A = M.baseline_matrix("c3", scale=0.05)
    perm = R.rcm_order(A)
    Ap = R.permute(A, perm)
    assert Ap.nnz == A.nnz and np.all(np.diff(Ap.indptr) >= 0)
    for r in range(0, Ap.rows, 97):  # columns sorted within each row
        seg = Ap.indices[Ap.indptr[r]:Ap.indptr[r + 1]]
        assert np.all(np.diff(seg) > 0)
    rng = np.random.default_rng(4)
    x = rng.uniform(-1, 1, A.cols)
    y = O.spmv(A, x)
    yp = O.spmv(Ap, R.permute_rows(x, perm))
    assert np.allclose(yp, y[perm], rtol=0, atol=1e-12 * max(1.0, np.abs(y).max()))
    B = rng.uniform(-1, 1, (A.cols, 5))
    C = O.spmm(A, B)
    Cp = O.spmm(Ap, R.permute_rows(B, perm))
    assert np.allclose(Cp, C[perm], rtol=0, atol=1e-12 * max(1.0, np.abs(C).max()))


def test_rcm_handles_components_empty_rows_and_self_loops():
    # two disjoint paths, an isolated node, a self loop, an empty row
    rows = [[1], [0, 2], [1], [3], [], [6], [5, 7], [6, 7]]
    indptr = np.zeros(len(rows) + 1, np.int64)
    np.cumsum([len(r) for r in rows], out=indptr[1:])
    idx = np.array([c for r in rows for c in r], np.int64)
    A = M.CSR(indptr, idx, np.ones(idx.size), (8, 8), "parts")
    perm = R.rcm_order(A)
    assert sorted(perm.tolist()) == list(range(8))
    # each path stays contiguous in the new numbering
    pos = R.inverse(perm)
    for comp in ([0, 1, 2], [5, 6, 7]):
        p = sorted(pos[comp])
        assert p[-1] - p[0] == 2


def test_rcm_rejects_bad_input():
    L = lib.load()
    ip = np.array([0, 1], np.int64)
    ix = np.array([3], np.int64)
    perm = np.empty(1, np.int64)
    assert L.tg_rcm_order(1, ip.ctypes.data, ix.ctypes.data, perm.ctypes.data) == lib.TG_EBOUNDS
    with pytest.raises(ValueError):
        R.rcm_order(M.CSR(np.array([0, 0], np.int64), np.zeros(0, np.int64), np.zeros(0), (1, 2), "rect"))


@pytest.mark.gpu
def test_reordered_spmm_on_the_gpu_matches_the_permuted_oracle():
    from tilegen_b200 import codegen as cg
    from tilegen_b200.verify import inputs_for, run_kernel

    A = R.scrambled(_band(20000, 4), seed=8)
    perm = R.rcm_order(A)
    Ap = R.permute(A, perm)
    data = inputs_for("spmm", A, 32, 3)
    ref = O.spmm(A, data[2])[perm]
    datap = (R.permute_rows(data[0], perm), R.permute_rows(data[1], perm), R.permute_rows(data[2], perm),
             R.permute_rows(data[3], perm), R.permute_rows(data[4], perm), data[5], data[6])
    out = run_kernel(cg.generate("spmm", cg.Config(split="merge", threads_per_row=8, vector_width=4)), Ap, datap, K=32)
    assert np.abs(out - ref).max() <= 1e-12 * np.abs(ref).max()
