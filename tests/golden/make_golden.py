"""Generate the golden fixtures in tests/golden/ from the reference itself.

Run where the reference tree is checked out (its location is taken from
TILEGEN_REFERENCE_ROOT, with the build container's mount point as the default):

    python tests/golden/make_golden.py

It imports the reference's Python package (tilegen.verify._inputs_for / _reference,
tilegen.matrices.make_matrix) and calls the reference's compiled CPU code
(oracle/_ref: cpp/src/ref.cpp and the OpenMP-emitted launchers, built by
oracle/build.py), and writes:

* ``kats.json``      -- the known-answer cases of cpp/tests/test_ref.cpp:25-116, with the
                        reference's serial C++ outputs.
* ``edge257.npz``    -- the reference GPU suite's 257x257 edge matrix
                        (tests/test_cuda_gpu.py:53-76), the verify inputs for it
                        (tilegen/verify.py:338-347, seed 7, K=8) and the reference outputs
                        of all five kernels: SciPy float64 (tilegen/verify.py:350-371),
                        the OpenMP backend in fp64 and in fp32.
* ``corner.npz``     -- the 4x4 / 3x3 / 2x2 cases of tests/test_verify.py:21-50 with
                        their SciPy reference outputs.
* ``corpus.json``    -- per corpus class (tilegen/matrices.py:164-178): shape, nnz,
                        digest, statistics, and SciPy reference SpMV/SpMM/SDDMM values at
                        sampled rows for the verify inputs.

The fixtures are small; none of them is read from the reference tree at test time.
"""

from __future__ import annotations

import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
# the reference checkout: $TILEGEN_REFERENCE_ROOT, else `reference` beside this repository
REF_ROOT = os.environ.get("TILEGEN_REFERENCE_ROOT", os.path.join(os.path.dirname(REPO), "reference"))


def main() -> int:
    sys.path.insert(0, REPO)
    from oracle import build as obuild
    from oracle import oracle as O
    from tilegen_b200 import matrices as M

    obuild.build_oracle()
    built = obuild.build_ref(REF_ROOT)
    if not built:
        raise SystemExit("reference tree not found at %s" % REF_ROOT)

    sys.path.insert(0, REF_ROOT)
    import scipy.sparse as sp
    from tilegen import matrices as RM  # reference
    from tilegen import verify as RV  # reference

    sys.path.insert(0, os.path.join(REF_ROOT, "tests"))
    import test_cuda_gpu as RT  # reference test module (its matrix builder)

    ref = O.ref_lib()
    P = O._ptr

    # ---------------------------------------------------------------- KATs
    kats = []

    def kat_spmv(name, rows, cols, ip, ix, d, x, expect):
        ip = np.asarray(ip, np.int64); ix = np.asarray(ix, np.int64)
        d = np.asarray(d, np.float64); x = np.asarray(x, np.float64)
        y = np.empty(rows)
        ref.tgref_spmv_f64(P(ip), P(ix), P(d), rows, cols, ix.size, P(x), P(y))
        assert np.allclose(y, expect), (name, y, expect)
        kats.append({"name": name, "op": "spmv", "rows": rows, "cols": cols, "indptr": ip.tolist(),
                     "indices": ix.tolist(), "data": d.tolist(), "x": x.tolist(), "expect": y.tolist()})

    kat_spmv("2x2 identity csr_spmv", 2, 2, [0, 1, 2], [0, 1], [1.0, 1.0], [3.0, -4.0], [3.0, -4.0])
    kat_spmv("empty row yields zero", 3, 3, [0, 1, 1, 2], [0, 2], [2.0, 5.0], [1.0, 1.0, 1.0], [2.0, 0.0, 5.0])
    kat_spmv("all-zero-data matrix yields zero", 2, 2, [0, 2, 3], [0, 1, 1], [0.0, 0.0, 0.0], [7.0, 9.0],
             [0.0, 0.0])
    # dense_spmv [1 2; 3 4] * [5; 6] = [17; 39], written as a full CSR
    kat_spmv("dense_spmv matches hand computation", 2, 2, [0, 2, 4], [0, 1, 0, 1], [1.0, 2.0, 3.0, 4.0],
             [5.0, 6.0], [17.0, 39.0])
    # csr_spmm small: A = [1 2; 0 3], B = I2 => C = A
    ip = np.array([0, 2, 3], np.int64); ix = np.array([0, 1, 1], np.int64); d = np.array([1.0, 2.0, 3.0])
    B = np.array([1.0, 0.0, 0.0, 1.0]); C = np.empty(4)
    ref.tgref_spmm_f64(P(ip), P(ix), P(d), 2, 2, 3, P(B), 2, P(C))
    assert np.allclose(C, [1, 2, 0, 3])
    kats.append({"name": "csr_spmm small", "op": "spmm", "rows": 2, "cols": 2, "K": 2, "indptr": ip.tolist(),
                 "indices": ix.tolist(), "data": d.tolist(), "B": B.tolist(), "expect": C.tolist()})
    # sddmm sampled product: A = I2, U = [[1,2],[3,4]], V = I2 => {1, 4}
    ip = np.array([0, 1, 2], np.int64); ix = np.array([0, 1], np.int64); d = np.array([1.0, 1.0])
    U = np.array([1.0, 2.0, 3.0, 4.0]); V = np.array([1.0, 0.0, 0.0, 1.0]); out = np.empty(2)
    ref.tgref_sddmm_f64(P(ip), P(ix), P(d), 2, 2, 2, P(U), P(V), 2, P(out))
    assert np.allclose(out, [1, 4])
    kats.append({"name": "sddmm sampled product", "op": "sddmm", "rows": 2, "cols": 2, "K": 2,
                 "indptr": ip.tolist(), "indices": ix.tolist(), "data": d.tolist(), "U": U.tolist(),
                 "V": V.tolist(), "expect": out.tolist()})
    # fused_spmv_axpy: A = [1 1; 0 1], x = [1; 2], w = [1; 1], alpha 2, beta 3 => [9; 7]
    ip = np.array([0, 2, 3], np.int64); ix = np.array([0, 1, 1], np.int64); d = np.array([1.0, 1.0, 1.0])
    x = np.array([1.0, 2.0]); w = np.array([1.0, 1.0]); z = np.empty(2)
    ref.tgref_fused_spmv_axpy_f64(P(ip), P(ix), P(d), 2, 2, 3, P(x), P(w), 2.0, 3.0, P(z))
    assert np.allclose(z, [9, 7])
    kats.append({"name": "fused_spmv_axpy", "op": "fused_spmv_axpy", "rows": 2, "cols": 2,
                 "indptr": ip.tolist(), "indices": ix.tolist(), "data": d.tolist(), "x": x.tolist(),
                 "w": w.tolist(), "alpha": 2.0, "beta": 3.0, "expect": z.tolist()})
    # float path: 2x2 identity, fp32
    ip = np.array([0, 1, 2], np.int64); ix = np.array([0, 1], np.int64)
    d32 = np.array([1.0, 1.0], np.float32); x32 = np.array([3.0, -4.0], np.float32); y32 = np.empty(2, np.float32)
    ref.tgref_spmv_f32(P(ip), P(ix), P(d32), 2, 2, 2, P(x32), P(y32))
    kats.append({"name": "float path produces same result", "op": "spmv_f32", "rows": 2, "cols": 2,
                 "indptr": ip.tolist(), "indices": ix.tolist(), "data": d32.tolist(), "x": x32.tolist(),
                 "expect": y32.astype(np.float64).tolist()})
    with open(os.path.join(HERE, "kats.json"), "w") as fh:
        json.dump({"source": "cpp/tests/test_ref.cpp:25-116, outputs of cpp/src/ref.cpp", "cases": kats},
                  fh, indent=1)

    # ---------------------------------------------------------------- edge257
    A = RT._cuda_matrix()
    mine = M.edge_matrix(257, 2024)
    assert np.array_equal(A.indptr, mine.indptr) and np.array_equal(A.indices, mine.indices) \
        and np.array_equal(A.data, mine.data), "edge_matrix does not reproduce the reference's"
    K = 8
    data = RV._inputs_for("spmv", A, K, 7)
    x, w, Bm, Um, Vm, alpha, beta = data
    outs = {k: np.asarray(RV._reference(k, A, data), dtype=np.float64)
            for k in ("spmv", "spmm", "sddmm", "fused_spmv_axpy", "axpy")}
    # the reference OpenMP backend on the same inputs (fp64 and fp32)
    libs = O.ref_omp_libs()
    M_, N_ = A.shape
    ip, ix, dv = A.indptr.astype(np.int64), A.indices.astype(np.int64), A.data.astype(np.float64)
    omp = {}
    for dtype, npdt in (("f64", np.float64), ("f32", np.float32)):
        dd = dv.astype(npdt)
        xx, ww, BB, UU, VV = (a.astype(npdt) for a in (x, w, Bm, Um, Vm))
        k = O.RefOmpKernel(libs["ref_omp_spmv_%s_T32U1" % dtype], "spmv")
        y = np.zeros(M_, npdt); k(ip, ix, dd, xx, y, M_, N_, ix.size); omp["spmv_" + dtype] = y
        k = O.RefOmpKernel(libs["ref_omp_spmm_%s_T32U1" % dtype], "spmm")
        Cc = np.zeros((M_, K), npdt); k(ip, ix, dd, BB, Cc, M_, N_, K, ix.size); omp["spmm_" + dtype] = Cc
        k = O.RefOmpKernel(libs["ref_omp_sddmm_%s_T32U1" % dtype], "sddmm")
        o = np.zeros(ix.size, npdt); k(ip, ix, dd, UU, VV, o, M_, N_, K, ix.size); omp["sddmm_" + dtype] = o
    for dtype, npdt in (("f64", np.float64), ("f32", np.float32)):
        dd, xx, ww = dv.astype(npdt), x.astype(npdt), w.astype(npdt)
        k = O.RefOmpKernel(libs["ref_omp_fused_spmv_axpy_%s_T32U1" % dtype], "fused_spmv_axpy", dtype)
        z = np.zeros(M_, npdt); k(ip, ix, dd, xx, ww, z, alpha, beta, M_, N_, ix.size)
        omp["fused_spmv_axpy_" + dtype] = z
        k = O.RefOmpKernel(libs["ref_omp_axpy_%s_T32U1" % dtype], "axpy", dtype)
        z = np.zeros(M_, npdt); k(xx, ww, z, alpha, beta, M_); omp["axpy_" + dtype] = z
    np.savez_compressed(
        os.path.join(HERE, "edge257.npz"),
        indptr=ip, indices=ix, data=dv, shape=np.array(A.shape, np.int64), K=np.int64(K),
        x=x, w=w, B=Bm, U=Um, V=Vm, alpha=np.float64(alpha), beta=np.float64(beta),
        **{"ref_" + k: v for k, v in outs.items()}, **{"omp_" + k: v for k, v in omp.items()})

    # ---------------------------------------------------------------- corner cases
    def csr(rows, cols, ip, ix, d):
        return sp.csr_matrix((np.asarray(d, np.float64), np.asarray(ix, np.int64), np.asarray(ip, np.int64)),
                             shape=(rows, cols))

    corners = {
        "bug4": csr(4, 4, [0, 2, 3, 5, 6], [0, 1, 2, 1, 2, 3], [1.0, 2.0, 3.0, 4.0, 5.0, 6.0]),
        "empty_row3": csr(3, 3, [0, 1, 1, 3], [0, 1, 2], [2.0, 4.0, 5.0]),
        "zeros2": csr(2, 2, [0, 2, 3], [0, 1, 1], [0.0, 0.0, 0.0]),
        "small3": csr(3, 3, [0, 2, 3, 3], [0, 1, 2], [1.0, 2.0, 3.0]),
    }
    arrs = {}
    for name, Am in corners.items():
        dat = RV._inputs_for("spmv", Am, 8, 7)
        arrs[name + "_indptr"] = Am.indptr.astype(np.int64)
        arrs[name + "_indices"] = Am.indices.astype(np.int64)
        arrs[name + "_data"] = Am.data.astype(np.float64)
        arrs[name + "_shape"] = np.array(Am.shape, np.int64)
        for k in ("spmv", "spmm", "sddmm", "fused_spmv_axpy", "axpy"):
            arrs[name + "_ref_" + k] = np.asarray(RV._reference(k, Am, dat), np.float64)
        for nm, v in zip(("x", "w", "B", "U", "V"), dat[:5]):
            arrs[name + "_" + nm] = v
    np.savez_compressed(os.path.join(HERE, "corner.npz"), **arrs)

    # ---------------------------------------------------------------- corpus
    corpus = {"seed": RM.SEED, "source": "tilegen/matrices.py:164-178; tilegen/verify.py:338-371", "classes": {}}
    for cls in RM.corpus_classes():
        Am = RM.make_matrix(cls)
        mm = M.CSR(Am.indptr.astype(np.int64), Am.indices.astype(np.int64), Am.data.astype(np.float64),
                   tuple(Am.shape), cls)
        dat = RV._inputs_for("spmv", Am, 8, 7)
        rng = np.random.default_rng(99)
        rows = np.unique(np.concatenate([[0, Am.shape[0] - 1], rng.integers(0, Am.shape[0], 62)]))
        y = np.asarray(RV._reference("spmv", Am, dat))[rows]
        Cm = np.asarray(RV._reference("spmm", Am, dat))[rows]
        sd = np.asarray(RV._reference("sddmm", Am, dat))
        pos = np.unique(rng.integers(0, Am.nnz, 64))
        corpus["classes"][cls] = {
            "shape": list(Am.shape), "nnz": int(Am.nnz), "digest": M.csr_digest(mm),
            "stats": M.matrix_stats(mm), "rows": rows.tolist(), "spmv": y.tolist(), "spmm": Cm.tolist(),
            "sddmm_pos": pos.tolist(), "sddmm": sd[pos].tolist(),
        }
    with open(os.path.join(HERE, "corpus.json"), "w") as fh:
        json.dump(corpus, fh, indent=1)
    print("golden fixtures written to", HERE)
    return 0


if __name__ == "__main__":
    sys.exit(main())
