"""The CPU oracle, pinned against the reference's own outputs (tests/golden)."""

from __future__ import annotations

import os

import numpy as np
import pytest

from oracle import build as obuild
from oracle import oracle as O
from tilegen_b200 import matrices as M


def test_known_answer_cases(kats):
    """cpp/tests/test_ref.cpp:25-116 through the C oracle."""
    assert len(kats) == 8
    for case in kats:
        ip, ix = np.array(case["indptr"], np.int64), np.array(case["indices"], np.int64)
        if case["op"] in ("spmv", "spmv_f32"):
            dt = np.float32 if case["op"] == "spmv_f32" else np.float64
            y = O.spmv((ip, ix, np.array(case["data"], dt)), np.array(case["x"], dt), dtype=dt)
            assert np.array_equal(y.astype(np.float64), np.array(case["expect"])), case["name"]
        elif case["op"] == "spmm":
            B = np.array(case["B"]).reshape(case["cols"], case["K"])
            C = O.spmm((ip, ix, np.array(case["data"])), B)
            assert np.array_equal(C.ravel(), np.array(case["expect"])), case["name"]
        elif case["op"] == "sddmm":
            U = np.array(case["U"]).reshape(case["rows"], case["K"])
            V = np.array(case["V"]).reshape(case["cols"], case["K"])
            out = O.sddmm((ip, ix, np.array(case["data"])), U, V)
            assert np.array_equal(out, np.array(case["expect"])), case["name"]
        elif case["op"] == "fused_spmv_axpy":
            z = O.fused_spmv_axpy((ip, ix, np.array(case["data"])), np.array(case["x"]), np.array(case["w"]),
                                  case["alpha"], case["beta"])
            assert np.array_equal(z, np.array(case["expect"])), case["name"]
        else:
            raise AssertionError(case["op"])


def test_edge_matrix_matches_scipy_reference_exactly(edge, edge_csr):
    """Row-ordered serial sums reproduce the reference's SciPy float64 outputs bit for
    bit for the row-reduction kernels (tilegen/verify.py:350-371)."""
    x, w, B, U, V = edge["x"], edge["w"], edge["B"], edge["U"], edge["V"]
    a, b = float(edge["alpha"]), float(edge["beta"])
    A = (edge_csr.indptr, edge_csr.indices, edge_csr.data)
    assert np.array_equal(O.spmv(A, x), edge["ref_spmv"])
    assert np.array_equal(O.fused_spmv_axpy(A, x, w, a, b), edge["ref_fused_spmv_axpy"])
    assert np.array_equal(O.axpy(x, w, a, b), edge["ref_axpy"])
    # SciPy's A @ B and numpy's einsum may reassociate inside a dot of length K
    np.testing.assert_allclose(O.spmm(A, B), edge["ref_spmm"], rtol=1e-14, atol=1e-13)
    np.testing.assert_allclose(O.sddmm(A, U, V), edge["ref_sddmm"], rtol=1e-14, atol=1e-13)


def test_edge_matrix_matches_reference_openmp_backend(edge, edge_csr):
    """The reference's OpenMP-emitted kernels (fp64 and fp32) on the same inputs."""
    A = (edge_csr.indptr, edge_csr.indices, edge_csr.data)
    x, w, B, U, V = edge["x"], edge["w"], edge["B"], edge["U"], edge["V"]
    # g++ -O3 -march=x86-64-v3 contracts the reference's multiply-adds into FMAs, so its
    # OpenMP build differs from the serial order by a few ulps (measured: 8.9e-16 abs)
    np.testing.assert_allclose(O.spmv(A, x), edge["omp_spmv_f64"], rtol=1e-13, atol=1e-14)
    np.testing.assert_allclose(O.spmm(A, B), edge["omp_spmm_f64"], rtol=1e-14, atol=1e-13)
    np.testing.assert_allclose(O.sddmm(A, U, V), edge["omp_sddmm_f64"], rtol=1e-14, atol=1e-13)
    f = np.float32
    A32 = (edge_csr.indptr, edge_csr.indices, edge_csr.data.astype(f))
    # g++ -O3 may contract the reference's fp32 multiply-adds into FMAs: compare at fp32 ulps
    np.testing.assert_allclose(O.spmv(A32, x.astype(f), dtype=f), edge["omp_spmv_f32"], rtol=2e-6, atol=2e-6)
    np.testing.assert_allclose(O.spmm(A32, B.astype(f), dtype=f), edge["omp_spmm_f32"], rtol=2e-6, atol=2e-6)
    np.testing.assert_allclose(O.sddmm(A32, U.astype(f), V.astype(f), dtype=f), edge["omp_sddmm_f32"],
                               rtol=2e-6, atol=2e-6)


def test_corner_cases(corner):
    for name in ("bug4", "empty_row3", "zeros2", "small3"):
        A = (corner[name + "_indptr"], corner[name + "_indices"], corner[name + "_data"])
        x = corner[name + "_x"]
        assert np.array_equal(O.spmv(A, x), corner[name + "_ref_spmv"]), name
    # all-zero data gives exact zeros (tests/test_verify.py:39-43)
    assert np.all(corner["zeros2_ref_spmv"] == 0.0)


def test_corpus_generator_and_oracle_match_reference(corpus):
    """make_matrix reproduces the reference corpus bit for bit (digests) and the oracle
    reproduces the reference's SpMV at sampled rows."""
    from tilegen_b200.verify import inputs_for

    for cls, info in corpus["classes"].items():
        m = M.make_matrix(cls)
        assert list(m.shape) == info["shape"] and m.nnz == info["nnz"], cls
        assert M.csr_digest(m) == info["digest"], cls
        x = inputs_for("spmv", m, 8, 7)[0]
        rows = np.array(info["rows"], np.int64)
        y = np.concatenate([O.spmv_rows(m, x, r, r + 1) for r in rows])
        assert np.array_equal(y, np.array(info["spmv"])), cls


@pytest.mark.skipif(not os.path.exists(obuild.TGREF_LIB), reason="reference C++ not built here")
def test_oracle_matches_reference_cpp(edge_csr, edge):
    """Same results as the reference's serial cpp/src/ref.cpp compiled from its tree."""
    ref = O.ref_lib()
    A = edge_csr
    P = O._ptr
    y = np.empty(A.rows)
    ref.tgref_spmv_f64(P(A.indptr), P(A.indices), P(A.data), A.rows, A.cols, A.nnz, P(edge["x"]), P(y))
    assert np.array_equal(y, O.spmv(A, edge["x"]))
    B = np.ascontiguousarray(edge["B"])
    C = np.empty((A.rows, 8))
    ref.tgref_spmm_f64(P(A.indptr), P(A.indices), P(A.data), A.rows, A.cols, A.nnz, P(B), 8, P(C))
    assert np.array_equal(C, O.spmm(A, B))
    U, V = np.ascontiguousarray(edge["U"]), np.ascontiguousarray(edge["V"])
    o = np.empty(A.nnz)
    ref.tgref_sddmm_f64(P(A.indptr), P(A.indices), P(A.data), A.rows, A.cols, A.nnz, P(U), P(V), 8, P(o))
    assert np.array_equal(o, O.sddmm(A, U, V))


def test_planted_bug_in_oracle_is_detected(edge, edge_csr):
    """The comparison catches a wrong result: drop the last row (the reference's
    inject_bug, tilegen/codegen.py:423-425) in an oracle output on the CPU."""
    from tilegen_b200.verify import tolerance

    y = O.spmv(edge_csr, edge["x"])
    y_bad = y.copy()
    y_bad[-1] = 0.0
    tol = tolerance(edge_csr, edge["ref_spmv"])
    assert np.abs(y - edge["ref_spmv"]).max() <= tol
    assert np.abs(y_bad - edge["ref_spmv"]).max() > tol


def test_power_iteration_oracle_matches_numpy():
    m = M.uniform_distinct(500, 500, 8, seed=3)
    S = m.to_scipy()
    x0 = np.random.default_rng(1).uniform(-1, 1, 500)
    x, nrm = O.power_iteration(m, x0, 5)
    z = x0.copy()
    for _ in range(5):
        yv = S @ z
        n = np.linalg.norm(yv)
        z = yv / n
    np.testing.assert_allclose(x, z, rtol=1e-12, atol=1e-14)
    assert abs(nrm - n) <= 1e-12 * n


def test_omp_spmv_matches_serial():
    m = M.baseline_matrix("c3", scale=0.05)
    x = np.random.default_rng(5).uniform(-1, 1, m.cols)
    y, threads = O.spmv_omp(m, x)
    assert threads >= 1
    assert np.array_equal(y, O.spmv(m, x))
