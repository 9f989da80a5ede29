"""Column-locality reordering: an optional preprocessing pass (no reference counterpart).

``rcm_order(A)`` is the reverse Cuthill-McKee order of a square matrix's symmetrised
pattern (``tg_rcm_order`` in libtilegen_b200.so, host code); ``permute(A, perm)`` applies
it to rows and columns together, ``A' = P A P^T`` with ``perm[new] = old``.  The dense
operands follow with ``permute_rows`` (``x' = P x``, ``B' = P B``, ``U' = P U``,
``V' = P V``), and the results come out permuted the same way (``y' = P y``,
``C' = P C``); SDDMM's values follow A's entries.  The point is the gathers: rows that
share columns get nearby numbers, so the dense rows they gather are reused while still
in L2.  A matrix whose columns are uniformly random has no such structure to find; a
banded or mesh matrix given in a scrambled numbering gets its band back.
"""

from __future__ import annotations

import ctypes

import numpy as np

from . import lib as _lib
from .matrices import CSR

__all__ = ["rcm_order", "inverse", "permute", "permute_rows", "bandwidth", "scrambled"]


def rcm_order(A: CSR) -> np.ndarray:
    """perm[new] = old: the reverse Cuthill-McKee order of a square A."""
    if A.rows != A.cols:
        raise ValueError("rcm_order needs a square matrix (got %dx%d)" % A.shape)
    ip = np.ascontiguousarray(A.indptr, np.int64)
    ix = np.ascontiguousarray(A.indices, np.int64)
    perm = np.empty(A.rows, np.int64)
    L = _lib.load()
    _lib.check(L.tg_rcm_order(A.rows, ip.ctypes.data, ix.ctypes.data if ix.size else None, perm.ctypes.data),
               "tg_rcm_order")
    return perm


def inverse(perm: np.ndarray) -> np.ndarray:
    inv = np.empty_like(perm)
    inv[perm] = np.arange(perm.size, dtype=perm.dtype)
    return inv


def permute(A: CSR, perm: np.ndarray) -> CSR:
    """A' = P A P^T: row k of A' is row perm[k] of A with every column j renamed inv[j];
    each row's columns sorted again (values follow them)."""
    n = A.rows
    if A.rows != A.cols or perm.size != n:
        raise ValueError("permute needs a square matrix and a permutation of its size")
    inv = inverse(perm)
    lens = np.diff(A.indptr)[perm]
    indptr = np.zeros(n + 1, np.int64)
    np.cumsum(lens, out=indptr[1:])
    # source position of every entry of A', row by row
    pos = np.repeat(A.indptr[:-1][perm] - indptr[:-1], lens) + np.arange(indptr[-1], dtype=np.int64)
    cols = inv[A.indices[pos]]
    vals = A.data[pos]
    rows = np.repeat(np.arange(n, dtype=np.int64), lens)
    order = np.argsort(rows * n + cols, kind="stable")
    return CSR(indptr, cols[order], vals[order], A.shape, "%s_rcm" % A.name)


def permute_rows(X: np.ndarray, perm: np.ndarray) -> np.ndarray:
    """X' = P X (row k of X' is row perm[k] of X)."""
    return np.ascontiguousarray(X[perm])


def bandwidth(A: CSR) -> int:
    """max |i - j| over the nonzeros."""
    if A.nnz == 0:
        return 0
    rows = np.repeat(np.arange(A.rows, dtype=np.int64), np.diff(A.indptr))
    return int(np.abs(rows - A.indices).max())


def scrambled(A: CSR, seed: int = 0) -> CSR:
    """A in a random symmetric numbering (what reordering is for: the same matrix with
    its locality hidden)."""
    perm = np.random.default_rng(seed).permutation(A.rows).astype(np.int64)
    m = permute(A, perm)
    return CSR(m.indptr, m.indices, m.data, m.shape, "%s_scrambled" % A.name)
