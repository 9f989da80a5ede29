/*
 * tg_oracle.c -- CPU restatement of TileGen's sparse kernels.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity oracle for the sm_100a kernels of
 * libtilegen_b200.so.  Only tests/, __graft_entry__.smoke() and the cpu_baseline /
 * reference legs of bench.py may load it, and only as the checker or the timed CPU
 * baseline; the product path never calls it.
 *
 * Each function restates the serial reference of TileGen (cpp/src/ref.cpp) in plain C:
 * rows in order, nonzeros of a row in index order, one accumulator per output.  That is
 * also the summation order of the SciPy float64 reference the reference's verify()
 * uses (tilegen/verify.py:350-371: A @ x, A @ B, einsum over A's pattern), so on x86-64
 * without FMA contraction the results agree bit for bit; tests/golden pins that.
 *
 * Build: oracle/build.py (gcc -O2 -ffp-contract=off -fopenmp -shared).
 */
#include <math.h>
#include <stddef.h>
#include <stdint.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* y = A x                                   (cpp/src/ref.cpp:6-15) */
void tgo_spmv_f64(const int64_t* indptr, const int64_t* indices, const double* data, const double* x,
                  double* y, int64_t rows) {
    for (int64_t i = 0; i < rows; ++i) {
        double acc = 0.0;
        for (int64_t p = indptr[i]; p < indptr[i + 1]; ++p) acc += data[p] * x[indices[p]];
        y[i] = acc;
    }
}

/* fp32 instantiation of the same loop      (cpp/src/ref.cpp:77-78) */
void tgo_spmv_f32(const int64_t* indptr, const int64_t* indices, const float* data, const float* x, float* y,
                  int64_t rows) {
    for (int64_t i = 0; i < rows; ++i) {
        float acc = 0.0f;
        for (int64_t p = indptr[i]; p < indptr[i + 1]; ++p) acc += data[p] * x[indices[p]];
        y[i] = acc;
    }
}

/* Row range [r0, r1) of SpMV, used by the multi-threaded CPU baseline below and by the
 * sampled-row checks of full-size workloads. */
void tgo_spmv_rows_f64(const int64_t* indptr, const int64_t* indices, const double* data, const double* x,
                       double* y, int64_t r0, int64_t r1) {
    for (int64_t i = r0; i < r1; ++i) {
        double acc = 0.0;
        for (int64_t p = indptr[i]; p < indptr[i + 1]; ++p) acc += data[p] * x[indices[p]];
        y[i - r0] = acc;
    }
}

/* OpenMP row-parallel SpMV: the same per-row arithmetic as tgo_spmv_f64, rows spread over
 * the host threads with the schedule the reference's OpenMP emitter uses
 * (tilegen/codegen.py:430, `schedule(dynamic, 256)`).  Returns the thread count used. */
int tgo_spmv_f64_omp(const int64_t* indptr, const int64_t* indices, const double* data, const double* x,
                     double* y, int64_t rows) {
    int nthreads = 1;
#pragma omp parallel
    {
#pragma omp single
        {
#ifdef _OPENMP
            nthreads = omp_get_num_threads();
#endif
        }
#pragma omp for schedule(dynamic, 256)
        for (int64_t i = 0; i < rows; ++i) {
            double acc = 0.0;
            for (int64_t p = indptr[i]; p < indptr[i + 1]; ++p) acc += data[p] * x[indices[p]];
            y[i] = acc;
        }
    }
    return nthreads;
}

/* C = A B, B is cols x K, C is rows x K     (cpp/src/ref.cpp:31-43) */
void tgo_spmm_f64(const int64_t* indptr, const int64_t* indices, const double* data, const double* B, double* C,
                  int64_t rows, int64_t K) {
    for (int64_t i = 0; i < rows; ++i) {
        double* c = C + i * K;
        for (int64_t k = 0; k < K; ++k) c[k] = 0.0;
        for (int64_t p = indptr[i]; p < indptr[i + 1]; ++p) {
            const double a = data[p];
            const double* b = B + indices[p] * K;
            for (int64_t k = 0; k < K; ++k) c[k] += a * b[k];
        }
    }
}

void tgo_spmm_f32(const int64_t* indptr, const int64_t* indices, const float* data, const float* B, float* C,
                  int64_t rows, int64_t K) {
    for (int64_t i = 0; i < rows; ++i) {
        float* c = C + i * K;
        for (int64_t k = 0; k < K; ++k) c[k] = 0.0f;
        for (int64_t p = indptr[i]; p < indptr[i + 1]; ++p) {
            const float a = data[p];
            const float* b = B + indices[p] * K;
            for (int64_t k = 0; k < K; ++k) c[k] += a * b[k];
        }
    }
}

/* out[p] = data[p] * sum_k U[i,k] V[j,k]    (cpp/src/ref.cpp:46-59) */
void tgo_sddmm_f64(const int64_t* indptr, const int64_t* indices, const double* data, const double* U,
                   const double* V, double* out, int64_t rows, int64_t K) {
    for (int64_t i = 0; i < rows; ++i) {
        for (int64_t p = indptr[i]; p < indptr[i + 1]; ++p) {
            const double* u = U + i * K;
            const double* v = V + indices[p] * K;
            double acc = 0.0;
            for (int64_t k = 0; k < K; ++k) acc += u[k] * v[k];
            out[p] = data[p] * acc;
        }
    }
}

void tgo_sddmm_f32(const int64_t* indptr, const int64_t* indices, const float* data, const float* U,
                   const float* V, float* out, int64_t rows, int64_t K) {
    for (int64_t i = 0; i < rows; ++i) {
        for (int64_t p = indptr[i]; p < indptr[i + 1]; ++p) {
            const float* u = U + i * K;
            const float* v = V + indices[p] * K;
            float acc = 0.0f;
            for (int64_t k = 0; k < K; ++k) acc += u[k] * v[k];
            out[p] = data[p] * acc;
        }
    }
}

/* z = alpha (A x) + beta w                  (cpp/src/ref.cpp:62-73) */
void tgo_fused_spmv_axpy_f64(const int64_t* indptr, const int64_t* indices, const double* data,
                             const double* x, const double* w, double* z, double alpha, double beta,
                             int64_t rows) {
    for (int64_t i = 0; i < rows; ++i) {
        double acc = 0.0;
        for (int64_t p = indptr[i]; p < indptr[i + 1]; ++p) acc += data[p] * x[indices[p]];
        z[i] = alpha * acc + beta * w[i];
    }
}

/* z = alpha x + beta w                      (tilegen/verify.py:369-370) */
void tgo_axpy_f64(const double* x, const double* w, double* z, double alpha, double beta, int64_t n) {
    for (int64_t i = 0; i < n; ++i) z[i] = alpha * x[i] + beta * w[i];
}

/* Power iteration x <- A x / ||A x||_2, `iters` times, in place on x (length rows == cols).
 * No counterpart in the reference (the multi-GPU mode is new); this is the float64
 * statement of the iteration the bench runs.  `y` is scratch of length rows.  Returns
 * the last norm ||A x_{k-1}||. */
double tgo_power_iteration_f64(const int64_t* indptr, const int64_t* indices, const double* data, double* x,
                               double* y, int64_t rows, int iters) {
    double nrm = 0.0;
    for (int it = 0; it < iters; ++it) {
        tgo_spmv_f64(indptr, indices, data, x, y, rows);
        double s = 0.0;
        for (int64_t i = 0; i < rows; ++i) s += y[i] * y[i];
        nrm = sqrt(s);
        const double inv = nrm > 0.0 ? 1.0 / nrm : 0.0;
        for (int64_t i = 0; i < rows; ++i) x[i] = y[i] * inv;
    }
    return nrm;
}
