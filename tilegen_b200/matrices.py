"""Deterministic sparse inputs for the b200 hot path.

Two generator families:

* **Reference corpus** (``make_matrix``): the six classes of TileGen's corpus
  (tilegen/matrices.py:164-178) -- banded, uniform_random, power_law, diagonal_heavy,
  dense_rows, blocked -- reproduced bit for bit.  Each class draws from its own numpy
  ``default_rng`` seeded with 1234 plus a fold of the class name, draws in the same order
  as the reference and canonicalises the COO triplets the same way (duplicates summed,
  indices sorted), because the published T4 numbers and the golden hashes in
  tests/golden refer to exactly those matrices.
* **BASELINE configurations** (``baseline_matrix``): C1..C5 of the benchmark contract --
  16 distinct sorted columns per row, the 7-diagonal band, Zipf(2) power-law rows
  rescaled to a target mean, the 8M-row / 32-per-row matrix of the multi-GPU power
  iteration (generated in independently seeded row blocks so every rank can build just
  its shard), and the 1M-row power-law matrix of SpMM/SDDMM.  Values are U(-1, 1).

All matrices are returned as :class:`CSR` with int64 ``indptr``/``indices``.
"""

from __future__ import annotations

import hashlib
import struct
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Tuple

import numpy as np

SEED = 1234  # seed of the reference corpus (tilegen/matrices.py:36)

__all__ = [
    "CSR",
    "make_matrix",
    "corpus_classes",
    "matrix_stats",
    "baseline_matrix",
    "baseline_configs",
    "uniform_distinct",
    "banded_clipped",
    "power_law_scaled",
    "c4_block_rows",
    "c4_rows",
    "edge_matrix",
    "csr_digest",
    "read_tgm1",
    "write_tgm1",
]


@dataclass
class CSR:
    """CSR matrix with int64 indices (the layout of the reference ABI)."""

    indptr: np.ndarray
    indices: np.ndarray
    data: np.ndarray
    shape: Tuple[int, int]
    name: str = "custom"
    meta: Dict[str, object] = field(default_factory=dict)

    @property
    def rows(self) -> int:
        return int(self.shape[0])

    @property
    def cols(self) -> int:
        return int(self.shape[1])

    @property
    def nnz(self) -> int:
        return int(self.indices.size)

    def astype(self, dtype) -> "CSR":
        return CSR(self.indptr, self.indices, self.data.astype(dtype), self.shape, self.name, dict(self.meta))

    def to_scipy(self):
        import scipy.sparse as sp

        m = sp.csr_matrix((self.data, self.indices, self.indptr), shape=self.shape)
        return m

    @staticmethod
    def from_scipy(m, name: str = "custom") -> "CSR":
        m = m.tocsr()
        return CSR(np.ascontiguousarray(m.indptr, dtype=np.int64), np.ascontiguousarray(m.indices, dtype=np.int64),
                   np.ascontiguousarray(m.data), tuple(int(s) for s in m.shape), name)

    def row_lengths(self) -> np.ndarray:
        return np.diff(self.indptr)


def _from_coo(rows: np.ndarray, cols: np.ndarray, vals: np.ndarray, shape, name: str) -> CSR:
    """Canonical CSR of COO triplets: duplicates summed, column indices sorted (the
    canonicalisation of tilegen/matrices.py:79-82, done with scipy as the reference does
    so that duplicate sums round identically)."""
    import scipy.sparse as sp

    m = sp.coo_matrix((vals, (rows, cols)), shape=shape).tocsr()
    m.sum_duplicates()
    m.sort_indices()
    return CSR.from_scipy(m, name)


# ----------------------------------------------------------------------------
# reference corpus (tilegen/matrices.py)
# ----------------------------------------------------------------------------
def _class_rng(name: str) -> np.random.Generator:
    """Per-class generator: SEED plus sum((position+1) * ord(char)) of the class name
    (tilegen/matrices.py:49-54)."""
    fold = 0
    for pos, ch in enumerate(name):
        fold += (pos + 1) * ord(ch)
    return np.random.default_rng(SEED + fold)


def _ref_banded(n: int, ndiag: int, name: str) -> CSR:
    """Band with `ndiag` diagonals, standard-normal values, +10 on the main diagonal;
    diagonals drawn from the lowest offset up (tilegen/matrices.py:57-76)."""
    rng = _class_rng(name)
    half = ndiag // 2
    rows_l, cols_l, vals_l = [], [], []
    for off in range(-half, half + 1):
        length = n - abs(off)
        v = rng.standard_normal(length)
        if off == 0:
            v = v + 10.0
        k = np.arange(length, dtype=np.int64)
        if off >= 0:
            r, c = k, k + off
        else:
            r, c = k - off, k
        rows_l.append(r)
        cols_l.append(c)
        vals_l.append(v)
    return _from_coo(np.concatenate(rows_l), np.concatenate(cols_l), np.concatenate(vals_l), (n, n), name)


def _ref_rows_from_counts(rng, counts: np.ndarray, ncols: int, n: int, name: str) -> CSR:
    rows = np.repeat(np.arange(n, dtype=np.int64), counts)
    cols = rng.integers(0, ncols, size=rows.size, dtype=np.int64)
    vals = rng.standard_normal(rows.size)
    return _from_coo(rows, cols, vals, (n, ncols), name)


def _ref_uniform(n: int, ncols: int, per_row: int, name: str) -> CSR:
    """`per_row` columns per row drawn with replacement (tilegen/matrices.py:85-94)."""
    rng = _class_rng(name)
    return _ref_rows_from_counts(rng, np.full(n, per_row, dtype=np.int64), ncols, n, name)


def _ref_power_law(n: int, ncols: int, alpha: float, cap: int, name: str) -> CSR:
    """Row lengths floor(u^(-1/(alpha-1))) (floor(1/u) for alpha = 2), clipped to
    [1, cap] (tilegen/matrices.py:97-114)."""
    rng = _class_rng(name)
    u = np.clip(rng.random(n), 1e-12, 1.0 - 1e-9)
    counts = np.floor(1.0 / u).astype(np.int64)
    if abs(alpha - 2.0) > 1e-9:
        counts = np.floor(np.power(u, -1.0 / (alpha - 1.0))).astype(np.int64)
    counts = np.minimum(np.clip(counts, 1, cap), ncols)
    return _ref_rows_from_counts(rng, counts, ncols, n, name)


def _ref_dense_rows(n: int, ncols: int, frac: float, big: int, small: int, name: str) -> CSR:
    """`small` nonzeros per row except round(frac*n) rows with `big`
    (tilegen/matrices.py:117-132)."""
    rng = _class_rng(name)
    counts = np.full(n, small, dtype=np.int64)
    n_big = max(1, int(round(frac * n)))
    counts[rng.choice(n, size=n_big, replace=False)] = big
    counts = np.minimum(counts, ncols)
    return _ref_rows_from_counts(rng, counts, ncols, n, name)


def _ref_blocked(n: int, bs: int, per_row: int, name: str) -> CSR:
    """Dense bs x bs blocks, the diagonal block plus random block columns per block row
    (tilegen/matrices.py:135-161).  The block-column set is iterated as a Python set,
    as the reference does, because that order decides which values land where."""
    if n % bs:
        raise ValueError("blocked matrix requires n divisible by block size")
    rng = _class_rng(name)
    nb = n // bs
    local = np.arange(bs, dtype=np.int64)
    rr_l, cc_l, vv_l = [], [], []
    for br in range(nb):
        bset = {br}
        while len(bset) < per_row:
            bset.add(int(rng.integers(0, nb)))
        for bc in bset:
            g_r, g_c = np.meshgrid(br * bs + local, bc * bs + local, indexing="ij")
            rr_l.append(g_r.ravel())
            cc_l.append(g_c.ravel())
            vv_l.append(rng.standard_normal(bs * bs))
    return _from_coo(np.concatenate(rr_l), np.concatenate(cc_l), np.concatenate(vv_l), (n, n), name)


def corpus_classes() -> List[str]:
    return ["banded", "uniform_random", "power_law", "diagonal_heavy", "dense_rows", "blocked"]


def make_matrix(class_name: str) -> CSR:
    """One class of the reference corpus (tilegen/matrices.py:164-178)."""
    if class_name == "banded":
        return _ref_banded(200000, 7, "banded")
    if class_name == "uniform_random":
        return _ref_uniform(100000, 100000, 16, "uniform_random")
    if class_name == "power_law":
        return _ref_power_law(100000, 100000, 2.0, 2000, "power_law")
    if class_name == "diagonal_heavy":
        return _ref_banded(200000, 3, "diagonal_heavy")
    if class_name == "dense_rows":
        return _ref_dense_rows(20000, 20000, 0.01, 2000, 4, "dense_rows")
    if class_name == "blocked":
        return _ref_blocked(100000, 8, 2, "blocked")
    raise ValueError("unknown matrix class: %s" % class_name)


def matrix_stats(m: CSR) -> Dict[str, object]:
    """Row-length statistics (the manifest fields of tilegen/matrices.py:192-212)."""
    counts = m.row_lengths().astype(np.float64)
    mean = float(counts.mean()) if counts.size else 0.0
    mx = float(counts.max()) if counts.size else 0.0
    return {
        "class_name": m.name,
        "rows": m.rows,
        "cols": m.cols,
        "nnz": m.nnz,
        "nnz_per_row_mean": mean,
        "nnz_per_row_median": float(np.median(counts)) if counts.size else 0.0,
        "nnz_per_row_max": mx,
        "nnz_per_row_stddev": float(counts.std()) if counts.size else 0.0,
        "imbalance_ratio": float(mx / mean) if mean > 0 else 0.0,
    }


def csr_digest(m: CSR) -> str:
    """sha256 over shape, indptr, indices and data bytes (little-endian int64/float)."""
    h = hashlib.sha256()
    h.update(np.asarray(m.shape, dtype="<i8").tobytes())
    h.update(np.ascontiguousarray(m.indptr, dtype="<i8").tobytes())
    h.update(np.ascontiguousarray(m.indices, dtype="<i8").tobytes())
    h.update(np.ascontiguousarray(m.data).astype(m.data.dtype.newbyteorder("<")).tobytes())
    return h.hexdigest()


# ----------------------------------------------------------------------------
# BASELINE configurations
# ----------------------------------------------------------------------------
def _sorted_uniform_ints(rng: np.random.Generator, nrows: int, per_row: int, ncols: int) -> np.ndarray:
    """Sorted iid uniform integers in [0, ncols): floor(ncols * U_(k)) where the order
    statistics U_(1) <= ... <= U_(per_row) of per_row uniforms are built directly as
    normalised partial sums of per_row + 1 standard exponentials (no sort needed)."""
    e = rng.standard_exponential(size=(nrows, per_row + 1))
    s = np.cumsum(e, axis=1)
    u = s[:, :per_row] / s[:, per_row:per_row + 1]
    return np.minimum(np.floor(u * ncols).astype(np.int64), ncols - 1)


def _distinct_sorted_rows(rng: np.random.Generator, nrows: int, per_row: int, ncols: int) -> np.ndarray:
    """(nrows, per_row) int64 array: each row `per_row` distinct columns drawn uniformly
    without replacement from [0, ncols), sorted.  Rows of iid uniform draws that contain
    a repeat are redrawn whole until every row is distinct; iid draws conditioned on
    being distinct are exactly uniform over per_row-subsets.  When repeats would be
    frequent (per_row^2 > ncols) rows are drawn one by one with rng.choice instead."""
    if per_row > ncols:
        raise ValueError("per_row > ncols")
    if per_row * per_row > ncols:
        out = np.empty((nrows, per_row), dtype=np.int64)
        for r in range(nrows):
            out[r] = np.sort(rng.choice(ncols, size=per_row, replace=False))
        return out
    out = _sorted_uniform_ints(rng, nrows, per_row, ncols)
    bad = np.nonzero((out[:, 1:] == out[:, :-1]).any(axis=1))[0] if per_row > 1 else np.array([], np.int64)
    while bad.size:
        redraw = _sorted_uniform_ints(rng, bad.size, per_row, ncols)
        out[bad] = redraw
        still = (redraw[:, 1:] == redraw[:, :-1]).any(axis=1)
        bad = bad[still]
    return out


def uniform_distinct(n: int, ncols: int, per_row: int, seed: int, name: str = "uniform_random") -> CSR:
    """C1: `per_row` distinct sorted columns per row, values U(-1, 1)."""
    rng = np.random.default_rng(seed)
    cols = _distinct_sorted_rows(rng, n, per_row, ncols).ravel()
    vals = rng.uniform(-1.0, 1.0, size=cols.size)
    indptr = np.arange(0, (n + 1) * per_row, per_row, dtype=np.int64)
    return CSR(indptr, cols, vals, (n, ncols), name, {"seed": seed, "per_row": per_row})


def banded_clipped(n: int, offsets=range(-3, 4), seed: int = 0, name: str = "banded") -> CSR:
    """C2: one nonzero on each diagonal offset in `offsets` (clipped at the edges),
    values U(-1, 1) in row-major order."""
    offs = np.asarray(sorted(offsets), dtype=np.int64)
    r = np.repeat(np.arange(n, dtype=np.int64), offs.size)
    c = r + np.tile(offs, n)
    keep = (c >= 0) & (c < n)
    r, c = r[keep], c[keep]
    rng = np.random.default_rng(seed)
    vals = rng.uniform(-1.0, 1.0, size=c.size)
    indptr = np.zeros(n + 1, dtype=np.int64)
    np.add.at(indptr, r + 1, 1)
    indptr = np.cumsum(indptr)
    return CSR(indptr, c, vals, (n, n), name, {"seed": seed, "offsets": [int(o) for o in offs]})


def _zipf_counts(rng: np.random.Generator, n: int, cap: int, target_mean: float, ncols: int) -> np.ndarray:
    """Zipf(alpha=2) row lengths by inverse transform floor(1/u) (the reference's
    power-law sampler, tilegen/matrices.py:100-107) clipped to [1, cap], then scaled by
    the factor s that brings the mean to `target_mean` (lengths round(s*k), at least 1;
    s found by bisection).  The realised mean/max are recorded by the caller."""
    u = np.clip(rng.random(n), 1e-12, 1.0 - 1e-9)
    k = np.clip(np.floor(1.0 / u), 1, cap)
    lo, hi = 0.0, 4.0 * target_mean
    for _ in range(60):
        s = 0.5 * (lo + hi)
        mean = np.maximum(1.0, np.floor(k * s + 0.5)).mean()
        if mean < target_mean:
            lo = s
        else:
            hi = s
    counts = np.maximum(1, np.floor(k * (0.5 * (lo + hi)) + 0.5)).astype(np.int64)
    return np.minimum(counts, ncols)


def power_law_scaled(n: int, ncols: int, target_mean: float, cap: int, seed: int, name: str = "power_law") -> CSR:
    """C3/C5: power-law row lengths (see _zipf_counts), columns uniform without
    replacement and sorted, values U(-1, 1)."""
    rng = np.random.default_rng(seed)
    counts = _zipf_counts(rng, n, cap, target_mean, ncols)
    indptr = np.zeros(n + 1, dtype=np.int64)
    np.cumsum(counts, out=indptr[1:])
    indices = np.empty(int(indptr[-1]), dtype=np.int64)
    # short rows: vectorised distinct draws grouped by length; long rows: rng.choice
    order = np.argsort(counts, kind="stable")
    sc = counts[order]
    bounds = np.flatnonzero(np.diff(sc)) + 1
    groups = np.split(order, bounds)
    for g in groups:
        L = int(counts[g[0]])
        if L <= 256:
            block = _distinct_sorted_rows(rng, g.size, L, ncols)
            starts = indptr[g]
            idx = starts[:, None] + np.arange(L, dtype=np.int64)[None, :]
            indices[idx.ravel()] = block.ravel()
        else:
            for r in g:
                s = indptr[r]
                indices[s:s + L] = np.sort(rng.choice(ncols, size=L, replace=False))
    vals = rng.uniform(-1.0, 1.0, size=indices.size)
    return CSR(indptr, indices, vals, (n, ncols), name,
               {"seed": seed, "target_mean": target_mean, "cap": cap,
                "realised_mean": float(counts.mean()), "realised_max": int(counts.max())})


# C4 is built in row blocks of C4_BLOCK rows, block b seeded with (seed, b), so that any
# row range (a rank's shard) can be generated without the rest of the matrix.
C4_BLOCK = 1 << 16


def c4_block_rows(b: int, n: int, per_row: int, seed: int) -> Tuple[np.ndarray, np.ndarray]:
    """Columns (rows_in_block, per_row) and values of C4 row block b."""
    r0 = b * C4_BLOCK
    nr = min(C4_BLOCK, n - r0)
    rng = np.random.default_rng([seed, b])
    cols = _distinct_sorted_rows(rng, nr, per_row, n)
    vals = rng.uniform(-1.0, 1.0, size=(nr, per_row))
    return cols, vals


def c4_rows(r0: int, r1: int, n: int = 8_000_000, per_row: int = 32, seed: int = 4) -> CSR:
    """Rows [r0, r1) of C4 (an n x n matrix, `per_row` distinct sorted columns per row,
    U(-1,1) values) as a (r1-r0) x n CSR."""
    nr = r1 - r0
    indices = np.empty(nr * per_row, dtype=np.int64)
    data = np.empty(nr * per_row, dtype=np.float64)
    b0, b1 = r0 // C4_BLOCK, (r1 - 1) // C4_BLOCK if r1 > r0 else -1
    for b in range(b0, b1 + 1):
        cols, vals = c4_block_rows(b, n, per_row, seed)
        lo = max(r0, b * C4_BLOCK)
        hi = min(r1, b * C4_BLOCK + cols.shape[0])
        src = slice(lo - b * C4_BLOCK, hi - b * C4_BLOCK)
        dst = slice((lo - r0) * per_row, (hi - r0) * per_row)
        indices[dst] = cols[src].ravel()
        data[dst] = vals[src].ravel()
    indptr = np.arange(0, (nr + 1) * per_row, per_row, dtype=np.int64)
    return CSR(indptr, indices, data, (nr, n), "c4_uniform32", {"seed": seed, "row0": r0, "n": n})


def baseline_configs() -> Dict[str, Dict[str, object]]:
    """The BASELINE.json configurations, by short name."""
    return {
        "c1": {"kind": "spmv", "desc": "uniform_random 100000^2, 16 distinct cols/row (1.6M nnz), fp64"},
        "c2": {"kind": "spmv", "desc": "banded 200000^2, offsets -3..+3 clipped (1399988 nnz), fp64"},
        "c3": {"kind": "spmv", "desc": "power_law 100000^2, Zipf(2) rows scaled to mean 8, fp64"},
        "c4": {"kind": "power", "desc": "8000000^2 uniform, 32 distinct cols/row (256M nnz), 20 power iterations"},
        "c5": {"kind": "spmm/sddmm", "desc": "1000000^2 Zipf(2) mean 16; SpMM K=128, SDDMM K=64, fp32"},
    }


def baseline_matrix(name: str, scale: float = 1.0) -> CSR:
    """A BASELINE configuration matrix; `scale` < 1 shrinks the row count (tests)."""
    if name == "c1":
        n = max(64, int(100000 * scale))
        return uniform_distinct(n, n, 16, seed=1001, name="c1_uniform_random")
    if name == "c2":
        n = max(64, int(200000 * scale))
        return banded_clipped(n, range(-3, 4), seed=1002, name="c2_banded")
    if name == "c3":
        n = max(64, int(100000 * scale))
        return power_law_scaled(n, n, 8.0, 20000, seed=1003, name="c3_power_law")
    if name == "c4":
        n = max(64, int(8_000_000 * scale))
        m = c4_rows(0, n, n=n)
        m.name = "c4_uniform32"
        return m
    if name == "c5":
        n = max(64, int(1_000_000 * scale))
        return power_law_scaled(n, n, 16.0, 20000, seed=1005, name="c5_power_law")
    raise ValueError("unknown baseline config %r" % name)


# ----------------------------------------------------------------------------
# test-suite matrices
# ----------------------------------------------------------------------------
def edge_matrix(rows: int = 257, seed: int = 2024) -> CSR:
    """The reference GPU suite's edge-case matrix (tests/test_cuda_gpu.py:53-76): square,
    row r empty when r % 37 == 0, else 1..24 distinct sorted columns drawn by
    rng.choice without replacement, standard-normal values; `rows` exceeds every tile
    and block size so an undersized launch grid leaves rows unwritten."""
    rng = np.random.default_rng(seed)
    indptr = [0]
    indices: List[int] = []
    data: List[float] = []
    for r in range(rows):
        k = 0 if r % 37 == 0 else int(rng.integers(1, 25))
        if k:
            indices.extend(int(c) for c in np.sort(rng.choice(rows, size=k, replace=False)))
            data.extend(float(v) for v in rng.standard_normal(k))
        indptr.append(len(indices))
    return CSR(np.asarray(indptr, dtype=np.int64), np.asarray(indices, dtype=np.int64),
               np.asarray(data, dtype=np.float64), (rows, rows), "edge%d" % rows)


# ----------------------------------------------------------------------------
# TGM1 binary format (tilegen/matrices.py:38-46, 240-252; cpp/src/harness.cpp:36-55)
# ----------------------------------------------------------------------------
TGM1_MAGIC = 0x54474D31


def write_tgm1(path: str, m: CSR) -> None:
    """Little-endian: u32 magic 'TGM1', i64 rows, cols, nnz, then indptr, indices (i64)
    and data (f64)."""
    with open(path, "wb") as fh:
        fh.write(struct.pack("<I", TGM1_MAGIC))
        fh.write(struct.pack("<qqq", m.rows, m.cols, m.nnz))
        fh.write(np.ascontiguousarray(m.indptr, dtype="<i8").tobytes())
        fh.write(np.ascontiguousarray(m.indices, dtype="<i8").tobytes())
        fh.write(np.ascontiguousarray(m.data, dtype="<f8").tobytes())


def read_tgm1(path: str, name: Optional[str] = None) -> CSR:
    with open(path, "rb") as fh:
        (magic,) = struct.unpack("<I", fh.read(4))
        if magic != TGM1_MAGIC:
            raise ValueError("%s: bad magic 0x%08x (expected TGM1)" % (path, magic))
        rows, cols, nnz = struct.unpack("<qqq", fh.read(24))
        if rows < 0 or cols < 0 or nnz < 0:
            raise ValueError("%s: negative header field" % path)
        indptr = np.frombuffer(fh.read(8 * (rows + 1)), dtype="<i8").astype(np.int64)
        indices = np.frombuffer(fh.read(8 * nnz), dtype="<i8").astype(np.int64)
        data = np.frombuffer(fh.read(8 * nnz), dtype="<f8").astype(np.float64)
    if indptr.size != rows + 1 or indices.size != nnz or data.size != nnz:
        raise ValueError("%s: truncated TGM1 file" % path)
    return CSR(indptr, indices, data, (int(rows), int(cols)), name or path)
