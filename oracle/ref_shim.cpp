// ref_shim.cpp -- C entry points over the reference's own serial C++ kernels.
//
// TEST INFRASTRUCTURE ONLY.  Compiled together with the reference's cpp/src/ref.cpp
// (read in place from the reference tree, never copied) into oracle/_ref/libtgref.so by
// oracle/build.py, so ctypes can call tilegen::csr_spmv / csr_spmm / sddmm /
// fused_spmv_axpy (cpp/include/tilegen/ref.hpp:18-41) on numpy buffers.  Used only to
// pin the C restatement in tg_oracle.c against the reference itself.
#include <cstdint>
#include <vector>

#include "tilegen/ref.hpp"

namespace {

template <typename T>
tilegen::Csr<T> make_csr(const int64_t* indptr, const int64_t* indices, const T* data, int64_t rows, int64_t cols,
                         int64_t nnz) {
    tilegen::Csr<T> A;
    A.rows = rows;
    A.cols = cols;
    A.indptr.assign(indptr, indptr + rows + 1);
    A.indices.assign(indices, indices + nnz);
    A.data.assign(data, data + nnz);
    return A;
}

template <typename T>
void copy_out(const std::vector<T>& v, T* out) {
    for (size_t i = 0; i < v.size(); ++i) out[i] = v[i];
}

template <typename T>
void spmv(const int64_t* ip, const int64_t* ix, const T* d, int64_t rows, int64_t cols, int64_t nnz, const T* x,
          T* y) {
    auto A = make_csr<T>(ip, ix, d, rows, cols, nnz);
    std::vector<T> xv(x, x + cols), yv;
    tilegen::csr_spmv(A, xv, yv);
    copy_out(yv, y);
}

template <typename T>
void spmm(const int64_t* ip, const int64_t* ix, const T* d, int64_t rows, int64_t cols, int64_t nnz, const T* B,
          int64_t K, T* C) {
    auto A = make_csr<T>(ip, ix, d, rows, cols, nnz);
    std::vector<T> Bv(B, B + cols * K), Cv;
    tilegen::csr_spmm(A, Bv, K, Cv);
    copy_out(Cv, C);
}

template <typename T>
void sddmm(const int64_t* ip, const int64_t* ix, const T* d, int64_t rows, int64_t cols, int64_t nnz, const T* U,
           const T* V, int64_t K, T* out) {
    auto A = make_csr<T>(ip, ix, d, rows, cols, nnz);
    std::vector<T> Uv(U, U + rows * K), Vv(V, V + cols * K), Ov;
    tilegen::sddmm(A, Uv, Vv, K, Ov);
    copy_out(Ov, out);
}

}  // namespace

extern "C" {

void tgref_spmv_f64(const int64_t* ip, const int64_t* ix, const double* d, int64_t rows, int64_t cols, int64_t nnz,
                    const double* x, double* y) {
    spmv<double>(ip, ix, d, rows, cols, nnz, x, y);
}
void tgref_spmv_f32(const int64_t* ip, const int64_t* ix, const float* d, int64_t rows, int64_t cols, int64_t nnz,
                    const float* x, float* y) {
    spmv<float>(ip, ix, d, rows, cols, nnz, x, y);
}
void tgref_spmm_f64(const int64_t* ip, const int64_t* ix, const double* d, int64_t rows, int64_t cols, int64_t nnz,
                    const double* B, int64_t K, double* C) {
    spmm<double>(ip, ix, d, rows, cols, nnz, B, K, C);
}
void tgref_spmm_f32(const int64_t* ip, const int64_t* ix, const float* d, int64_t rows, int64_t cols, int64_t nnz,
                    const float* B, int64_t K, float* C) {
    spmm<float>(ip, ix, d, rows, cols, nnz, B, K, C);
}
void tgref_sddmm_f64(const int64_t* ip, const int64_t* ix, const double* d, int64_t rows, int64_t cols,
                     int64_t nnz, const double* U, const double* V, int64_t K, double* out) {
    sddmm<double>(ip, ix, d, rows, cols, nnz, U, V, K, out);
}
void tgref_sddmm_f32(const int64_t* ip, const int64_t* ix, const float* d, int64_t rows, int64_t cols, int64_t nnz,
                     const float* U, const float* V, int64_t K, float* out) {
    sddmm<float>(ip, ix, d, rows, cols, nnz, U, V, K, out);
}
void tgref_fused_spmv_axpy_f64(const int64_t* ip, const int64_t* ix, const double* d, int64_t rows, int64_t cols,
                               int64_t nnz, const double* x, const double* w, double alpha, double beta, double* z) {
    auto A = make_csr<double>(ip, ix, d, rows, cols, nnz);
    std::vector<double> xv(x, x + cols), wv(w, w + rows), zv;
    tilegen::fused_spmv_axpy(A, xv, wv, alpha, beta, zv);
    copy_out(zv, z);
}
void tgref_dense_spmv_f64(const double* A, int64_t m, int64_t n, const double* x, double* y) {
    std::vector<double> Av(A, A + m * n), xv(x, x + n), yv;
    tilegen::dense_spmv(Av, m, n, xv, yv);
    copy_out(yv, y);
}

}  // extern "C"
