"""Randomised checks of the oracle against SciPy/numpy float64 on ragged matrices (empty
rows, empty columns, one long row, a zero-row and a zero-column shape), beside the golden
fixtures of test_oracle.py."""

from __future__ import annotations

import numpy as np
import pytest

from oracle import oracle as O
from tilegen_b200.matrices import CSR


def _ragged(seed: int, rows: int, cols: int) -> CSR:
    rng = np.random.default_rng(seed)
    lens = rng.integers(0, 6, rows)
    if rows > 3:
        lens[rng.integers(0, rows)] = min(cols, 300)  # one long row
        lens[: rows // 4] = 0                         # a block of empty rows
    lens = np.minimum(lens, cols)
    indptr = np.zeros(rows + 1, np.int64)
    np.cumsum(lens, out=indptr[1:])
    idx = [np.sort(rng.choice(cols, size=L, replace=False)) for L in lens]
    indices = np.concatenate(idx).astype(np.int64) if rows else np.zeros(0, np.int64)
    return CSR(indptr, indices, rng.uniform(-1, 1, indices.size), (rows, cols), "ragged%d" % seed)


def _tol(ref, nnz_row):
    return 8 * np.finfo(np.float64).eps * max(1, nnz_row) * max(np.abs(ref).max(initial=0.0), 1.0) + 1e-12


@pytest.mark.parametrize("seed,rows,cols", [(1, 50, 40), (2, 400, 700), (3, 1, 1), (4, 0, 5), (5, 7, 0),
                                            (6, 1000, 1000)])
def test_oracle_kernels_match_scipy(seed, rows, cols):
    m = _ragged(seed, rows, cols)
    S = m.to_scipy()
    rng = np.random.default_rng(100 + seed)
    x, w = rng.standard_normal(cols), rng.standard_normal(rows)
    B, V, U = rng.standard_normal((cols, 8)), rng.standard_normal((cols, 8)), rng.standard_normal((rows, 8))
    longest = int(np.diff(m.indptr).max()) if rows else 0
    ref = S @ x
    assert np.abs(O.spmv(m, x) - ref).max(initial=0.0) <= _tol(ref, longest)
    assert np.abs(O.spmv_omp(m, x)[0] - ref).max(initial=0.0) <= _tol(ref, longest)
    refm = S @ B
    assert np.abs(O.spmm(m, B) - refm).max(initial=0.0) <= _tol(refm, longest)
    rr = np.repeat(np.arange(rows), np.diff(m.indptr))
    refs = m.data * np.einsum("ik,ik->i", U[rr], V[m.indices]) if m.nnz else np.zeros(0)
    assert np.abs(O.sddmm(m, U, V) - refs).max(initial=0.0) <= _tol(refs, 8)
    reff = 0.7 * ref - 1.3 * w
    assert np.abs(O.fused_spmv_axpy(m, x, w, 0.7, -1.3) - reff).max(initial=0.0) <= _tol(reff, longest)
