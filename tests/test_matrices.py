"""Input generators: BASELINE configurations, shard reproducibility, formats."""

from __future__ import annotations

import numpy as np

from tilegen_b200 import matrices as M


def _rows_strictly_increasing(m):
    for r in range(m.rows):
        seg = m.indices[m.indptr[r]:m.indptr[r + 1]]
        if seg.size > 1 and not np.all(np.diff(seg) > 0):
            return False
    return True


def test_c1_distinct_sorted_columns():
    m = M.baseline_matrix("c1", scale=0.02)
    assert m.nnz == 16 * m.rows
    assert _rows_strictly_increasing(m)
    assert m.indices.min() >= 0 and m.indices.max() < m.cols
    assert np.all((m.data >= -1) & (m.data < 1))


def test_c2_band_nnz_formula():
    m = M.baseline_matrix("c2")
    assert m.shape == (200000, 200000) and m.nnz == 1399988
    assert _rows_strictly_increasing(M.banded_clipped(50, range(-3, 4)))


def test_c3_power_law_targets():
    m = M.baseline_matrix("c3", scale=0.2)
    L = m.row_lengths()
    assert abs(L.mean() - 8.0) < 0.05
    assert L.max() > 50 * L.mean()
    assert _rows_strictly_increasing(m)


def test_c4_shards_are_slices_of_the_whole():
    n = 3 * M.C4_BLOCK + 1000
    whole = M.c4_rows(0, n, n=n, per_row=8, seed=9)
    a, b = M.C4_BLOCK - 10, 2 * M.C4_BLOCK + 7
    part = M.c4_rows(a, b, n=n, per_row=8, seed=9)
    assert np.array_equal(part.indices, whole.indices[a * 8:b * 8])
    assert np.array_equal(part.data, whole.data[a * 8:b * 8])
    assert np.array_equal(part.indptr, np.arange(0, (b - a + 1) * 8, 8))


def test_edge_matrix_structure(edge):
    m = M.edge_matrix()
    assert np.array_equal(m.indptr, edge["indptr"]) and np.array_equal(m.indices, edge["indices"])
    L = m.row_lengths()
    assert np.all(L[::37] == 0) and L.max() <= 24


def test_tgm1_roundtrip(tmp_path):
    m = M.baseline_matrix("c3", scale=0.01)
    p = str(tmp_path / "m.bin")
    M.write_tgm1(p, m)
    r = M.read_tgm1(p)
    assert r.shape == m.shape and np.array_equal(r.indptr, m.indptr) and np.array_equal(r.data, m.data)
    raw = open(p, "rb").read()
    assert raw[:4] == (0x54474D31).to_bytes(4, "little")


def test_matrix_stats_fields():
    s = M.matrix_stats(M.make_matrix("dense_rows"))
    assert s["imbalance_ratio"] > 10  # tests/test_env_matrices.py of the reference
