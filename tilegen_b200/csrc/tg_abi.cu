// C ABI of libtilegen_b200.so: argument checking, schedule resolution, the native
// tg_* entry points and the reference-compatible launch_* launchers.
//
// The launch_* functions replace the emitted launchers of the reference
// (tilegen/codegen.py:764-799 _launch_wrapper, signatures from _abi at :226-280) with
// the same argument lists and the same synchronous, default-stream behaviour.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <atomic>
#include <mutex>
#include <vector>

#include "tg_dense_host.cuh"
#include "tg_split.cuh"

namespace tg {

// ------------------------------------------------------------------ errors
namespace {
thread_local char t_msg[512] = "";
thread_local int t_last_status = TG_OK;
}  // namespace

int set_error(int status, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(t_msg, sizeof(t_msg), fmt, ap);
    va_end(ap);
    return status;
}

int check_cuda(cudaError_t e, const char* what) {
    if (e == cudaSuccess) return TG_OK;
    return set_error(TG_ECUDA, "%s: CUDA error %d (%s)", what, (int)e, cudaGetErrorString(e));
}

// Every kernel launch site calls check_launch right after its <<<...>>>, so this is
// also where launches are counted (tg_launch_count).
std::atomic<uint64_t> g_launches{0};

int check_launch(const char* what) {
    g_launches.fetch_add(1, std::memory_order_relaxed);
    return check_cuda(cudaGetLastError(), what);
}

// kernels defined in tg_spmv.cu
template <typename T, bool AXPY>
int spmv_run(const tg_csr& A, const T* x, T* y, const Epi<T, AXPY>& epi, const tg_sched& s, void* ws,
             size_t ws_bytes, cudaStream_t st);
size_t spmv_ws_bytes(int64_t rows, int64_t nnz, const tg_sched& s, size_t elem);
template <typename T>
int axpy_run(const T* x, const T* w, T* z, T alpha, T beta, int64_t n, int block, cudaStream_t st);
// power iteration (tg_power.cu)
size_t power_ws_bytes(int64_t nnz, const tg_sched& s);
int power_step_run(const tg_csr& A, const double* x, int nparts, int64_t stride, double* y, const tg_sched& s,
                   void* ws, size_t ws_bytes, cudaStream_t st);
int shard_norm2_run(double* shard, int64_t rows, int64_t stride, void* ws, size_t ws_bytes, cudaStream_t st);
int power_finalize_run(const double* x, int nparts, int64_t stride, int part, int64_t rows, double* x_out,
                       double* lambda_out, cudaStream_t st);
int power_step_p2p_run(const tg_csr& A, const double* x, int nparts, int rank, int64_t stride,
                       double* const* y_peers, unsigned long long* const* flag_peers, unsigned long long epoch,
                       const tg_sched& s, void* ws, size_t ws_bytes, cudaStream_t st);
size_t power_err_offset();
int power_step_ce_run(const tg_csr& A, const double* x, int nparts, int rank, int64_t stride, double* const* y_peers,
                      unsigned long long* const* flag_peers, unsigned long long epoch, int nchunks, const tg_sched& s,
                      void* ws, size_t ws_bytes, cudaStream_t st);
int p2p_wait_run(const unsigned long long* flag_local, int nparts, unsigned long long epoch, void* ws,
                 size_t ws_bytes, cudaStream_t st);

// ------------------------------------------------------------------ bounds check
// Sets bits of *err: 1 indptr[0] != 0, 2 indptr decreasing, 4 indptr[rows] != nnz,
// 8 column index outside [0, cols).
__global__ void csr_check_kernel(const int64_t* __restrict__ indptr, const int64_t* __restrict__ indices,
                                 int64_t rows, int64_t cols, int64_t nnz, uint32_t* err) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    uint32_t e = 0;
    if (tid == 0) {
        if (indptr[0] != 0) e |= 1u;
        if (indptr[rows] != nnz) e |= 4u;
    }
    for (int64_t r = tid; r < rows; r += stride)
        if (indptr[r + 1] < indptr[r]) e |= 2u;
    for (int64_t p = tid; p < nnz; p += stride) {
        const int64_t c = indices[p];
        if (c < 0 || c >= cols) e |= 8u;
    }
    if (e) atomicOr(err, e);
}

namespace {

std::mutex g_mu;
std::mutex g_shim_mu;  // launch_* share one workspace per device: one call at a time
tg_sched g_sched = {32, 1, 1, 1, 128, TG_SPLIT_ROWWISE, 0, 0u};

struct DeviceScratch {
    void* ws = nullptr;  // workspace cache of the launch_* launchers (grow-only)
    size_t ws_bytes = 0;
    uint32_t* err = nullptr;  // bounds-check word
};
std::vector<DeviceScratch> g_dev;

DeviceScratch* device_scratch() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return nullptr;
    if ((int)g_dev.size() <= dev) g_dev.resize(dev + 1);
    return &g_dev[dev];
}

}  // namespace

// Fills *out from `in` (NULL: the process schedule of tg_set_schedule) with every zero
// knob replaced by its default, and checks it.  Every tg_* entry point resolves its
// schedule here.
int resolve_schedule(const tg_sched* in, tg_sched* out) {
    tg_sched s;
    if (in) {
        s = *in;
    } else {
        std::lock_guard<std::mutex> lk(g_mu);
        s = g_sched;
    }
    if (s.tile <= 0) s.tile = 32;
    if (s.threads_per_row <= 0) s.threads_per_row = 1;
    if (s.unroll <= 0) s.unroll = 1;
    if (s.vector_width <= 0) s.vector_width = 1;
    if (s.block_size <= 0) s.block_size = 128;
    // AUTO: the host does not see the row lengths, so take the mapping that is
    // load-balanced for every distribution (rowwise is the tuned choice for regular rows)
    if (s.split == TG_SPLIT_AUTO) s.split = TG_SPLIT_MERGE;
    const int tpr = s.threads_per_row;
    if (tpr != 1 && tpr != 2 && tpr != 4 && tpr != 8 && tpr != 16 && tpr != 32)
        return set_error(TG_EINVAL, "threads_per_row must be 1, 2, 4, 8, 16 or 32 (got %d)", tpr);
    if (s.unroll != 1 && s.unroll != 2 && s.unroll != 4 && s.unroll != 8)
        return set_error(TG_EINVAL, "unroll must be 1, 2, 4 or 8 (got %d)", s.unroll);
    if (s.vector_width != 1 && s.vector_width != 2 && s.vector_width != 4)
        return set_error(TG_EINVAL, "vector_width must be 1, 2 or 4 (got %d)", s.vector_width);
    // the row kernels are compiled for at most 512 threads per CTA (up to 128 registers a
    // thread, so no instance spills); the reference's space tops out at 512 too
    if (s.block_size < 32 || s.block_size > 512 || s.block_size % 32 != 0)
        return set_error(TG_EINVAL, "block_size must be a multiple of 32 in [32, 512] (got %d)", s.block_size);
    if (s.block_size % tpr != 0)
        return set_error(TG_EINVAL, "block_size (%d) not divisible by threads_per_row (%d)", s.block_size, tpr);
    if (s.split != TG_SPLIT_ROWWISE && s.split != TG_SPLIT_MERGE && s.split != TG_SPLIT_STREAM &&
        s.split != TG_SPLIT_BLOCK)
        return set_error(TG_EINVAL, "split must be TG_SPLIT_ROWWISE, _MERGE, _STREAM, _BLOCK or _AUTO (got %d)",
                         s.split);
    if (s.chunk_nnz < 0) return set_error(TG_EINVAL, "chunk_nnz must be >= 0 (got %d)", s.chunk_nnz);
    *out = s;
    return TG_OK;
}

namespace {

int resolve(const tg_sched* in, tg_sched* out) { return resolve_schedule(in, out); }

int check_csr(const tg_csr* A, const char* op) {
    if (!A) return set_error(TG_EINVAL, "%s: null CSR descriptor", op);
    if (A->rows < 0 || A->cols < 0 || A->nnz < 0)
        return set_error(TG_EINVAL, "%s: negative size (rows=%lld cols=%lld nnz=%lld)", op, (long long)A->rows,
                         (long long)A->cols, (long long)A->nnz);
    if (!A->indptr) return set_error(TG_EINVAL, "%s: null indptr", op);
    if (A->nnz > 0 && (!A->indices || !A->data)) return set_error(TG_EINVAL, "%s: null indices/data", op);
    return TG_OK;
}

// Bounds-checked calls validate the CSR structure first and are synchronous on `st`.
int bounds_check(const tg_csr& A, cudaStream_t st) {
    uint32_t* err = nullptr;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        DeviceScratch* d = device_scratch();
        if (!d) return set_error(TG_ECUDA, "cudaGetDevice failed");
        if (!d->err) {
            int rc = check_cuda(cudaMalloc(&d->err, sizeof(uint32_t)), "cudaMalloc(bounds word)");
            if (rc != TG_OK) return rc;
        }
        err = d->err;
    }
    int rc = check_cuda(cudaMemsetAsync(err, 0, sizeof(uint32_t), st), "cudaMemsetAsync");
    if (rc != TG_OK) return rc;
    int64_t blocks = std::min<int64_t>(ceil_div(std::max(A.rows, A.nnz) + 1, 256), 148 * 16);
    csr_check_kernel<<<(unsigned)blocks, 256, 0, st>>>(A.indptr, A.indices, A.rows, A.cols, A.nnz, err);
    rc = check_launch("csr_check_kernel");
    if (rc != TG_OK) return rc;
    uint32_t h = 0;
    rc = check_cuda(cudaMemcpyAsync(&h, err, sizeof(h), cudaMemcpyDeviceToHost, st), "cudaMemcpyAsync");
    if (rc != TG_OK) return rc;
    rc = check_cuda(cudaStreamSynchronize(st), "cudaStreamSynchronize");
    if (rc != TG_OK) return rc;
    if (h)
        return set_error(TG_EBOUNDS, "CSR check failed (flags 0x%x:%s%s%s%s)", h, (h & 1) ? " indptr[0]!=0" : "",
                         (h & 2) ? " indptr decreasing" : "", (h & 4) ? " indptr[rows]!=nnz" : "",
                         (h & 8) ? " column index out of range" : "");
    return TG_OK;
}

void* shim_workspace(size_t need, int* rc) {
    *rc = TG_OK;
    if (need == 0) return nullptr;
    std::lock_guard<std::mutex> lk(g_mu);
    DeviceScratch* d = device_scratch();
    if (!d) {
        *rc = set_error(TG_ECUDA, "cudaGetDevice failed");
        return nullptr;
    }
    if (d->ws_bytes < need) {
        if (d->ws) cudaFree(d->ws);
        d->ws = nullptr;
        d->ws_bytes = 0;
        *rc = check_cuda(cudaMalloc(&d->ws, need), "cudaMalloc(launcher workspace)");
        if (*rc != TG_OK) return nullptr;
        d->ws_bytes = need;
    }
    return d->ws;
}

}  // namespace
}  // namespace tg

using namespace tg;

extern "C" {

const char* tg_version(void) { return "tilegen_b200 0.1.0 (sm_100a)"; }

const char* tg_last_error_string(void) { return t_msg; }

int tg_last_status(void) { return t_last_status; }

uint64_t tg_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

void tg_default_schedule(tg_sched* s) {
    if (s) *s = tg_sched{32, 1, 1, 1, 128, TG_SPLIT_ROWWISE, 0, 0u};
}

int tg_validate_schedule(const tg_sched* s) {
    if (!s) return set_error(TG_EINVAL, "null schedule");
    tg_sched out;
    return resolve(s, &out);
}

int tg_set_schedule(const tg_sched* s) {
    if (!s) return set_error(TG_EINVAL, "null schedule");
    tg_sched out;
    int rc = resolve(s, &out);
    if (rc != TG_OK) return rc;
    std::lock_guard<std::mutex> lk(g_mu);
    g_sched = *s;
    return TG_OK;
}

int tg_get_schedule(tg_sched* s) {
    if (!s) return set_error(TG_EINVAL, "null schedule");
    std::lock_guard<std::mutex> lk(g_mu);
    *s = g_sched;
    return TG_OK;
}

size_t tg_spmv_workspace_bytes(int64_t rows, int64_t nnz, const tg_sched* s) {
    tg_sched r;
    if (resolve(s, &r) != TG_OK) return 0;
    return spmv_ws_bytes(rows, nnz, r, sizeof(double));
}

size_t tg_spmm_workspace_bytes(int64_t rows, int64_t nnz, int64_t k, const tg_sched* s) {
    tg_sched r;
    if (resolve(s, &r) != TG_OK) return 0;
    // sized for fp64 partials, which also covers fp32
    return dense_ws_bytes<double>(rows, nnz, k, r, true) + dense_ws_bytes<float>(rows, nnz, k, r, true);
}

size_t tg_sddmm_workspace_bytes(int64_t rows, int64_t nnz, int64_t k, const tg_sched* s) {
    tg_sched r;
    if (resolve(s, &r) != TG_OK) return 0;
    return dense_ws_bytes<double>(rows, nnz, k, r, false);
}

#define TG_PRELUDE(op)                                     \
    tg_sched sc;                                           \
    int rc = resolve(s, &sc);                              \
    if (rc != TG_OK) return rc;                            \
    rc = check_csr(A, op);                                 \
    if (rc != TG_OK) return rc;                            \
    cudaStream_t st = static_cast<cudaStream_t>(stream);   \
    if ((sc.flags & TG_FLAG_INDEX32) &&                    \
        (strncmp(op, "tg_power", 8) != 0 || (sc.flags & TG_FLAG_BOUNDS_CHECK))) \
        return set_error(TG_EUNSUPPORTED, "%s: 32-bit column indices are taken by the power steps only, without bounds checking", op); \
    if (sc.flags & TG_FLAG_BOUNDS_CHECK) {                 \
        rc = bounds_check(*A, st);                         \
        if (rc != TG_OK) return rc;                        \
    }

int tg_spmv_f64(const tg_csr* A, const double* x, double* y, const tg_sched* s, void* workspace,
                size_t workspace_bytes, tg_stream_t stream) {
    TG_PRELUDE("tg_spmv_f64");
    if (A->rows > 0 && !y) return set_error(TG_EINVAL, "tg_spmv_f64: null y");
    if (A->nnz > 0 && !x) return set_error(TG_EINVAL, "tg_spmv_f64: null x");
    return spmv_run<double, false>(*A, x, y, Epi<double, false>{nullptr, 0.0, 0.0}, sc, workspace, workspace_bytes,
                                   st);
}

int tg_spmv_f32(const tg_csr* A, const float* x, float* y, const tg_sched* s, void* workspace,
                size_t workspace_bytes, tg_stream_t stream) {
    TG_PRELUDE("tg_spmv_f32");
    if (A->rows > 0 && !y) return set_error(TG_EINVAL, "tg_spmv_f32: null y");
    if (A->nnz > 0 && !x) return set_error(TG_EINVAL, "tg_spmv_f32: null x");
    return spmv_run<float, false>(*A, x, y, Epi<float, false>{nullptr, 0.f, 0.f}, sc, workspace, workspace_bytes, st);
}

int tg_fused_spmv_axpy_f64(const tg_csr* A, const double* x, const double* w, double* z, double alpha,
                           double beta, const tg_sched* s, void* workspace, size_t workspace_bytes,
                           tg_stream_t stream) {
    TG_PRELUDE("tg_fused_spmv_axpy_f64");
    if (A->rows > 0 && (!z || !w)) return set_error(TG_EINVAL, "tg_fused_spmv_axpy_f64: null w/z");
    if (A->nnz > 0 && !x) return set_error(TG_EINVAL, "tg_fused_spmv_axpy_f64: null x");
    return spmv_run<double, true>(*A, x, z, Epi<double, true>{w, alpha, beta}, sc, workspace, workspace_bytes, st);
}

int tg_fused_spmv_axpy_f32(const tg_csr* A, const float* x, const float* w, float* z, float alpha, float beta,
                           const tg_sched* s, void* workspace, size_t workspace_bytes, tg_stream_t stream) {
    TG_PRELUDE("tg_fused_spmv_axpy_f32");
    if (A->rows > 0 && (!z || !w)) return set_error(TG_EINVAL, "tg_fused_spmv_axpy_f32: null w/z");
    if (A->nnz > 0 && !x) return set_error(TG_EINVAL, "tg_fused_spmv_axpy_f32: null x");
    return spmv_run<float, true>(*A, x, z, Epi<float, true>{w, alpha, beta}, sc, workspace, workspace_bytes, st);
}

int tg_spmm_f32(const tg_csr* A, const float* B, float* C, int64_t k, const tg_sched* s, void* workspace,
                size_t workspace_bytes, tg_stream_t stream) {
    TG_PRELUDE("tg_spmm_f32");
    if (A->rows > 0 && !C) return set_error(TG_EINVAL, "tg_spmm_f32: null C");
    if (A->nnz > 0 && !B) return set_error(TG_EINVAL, "tg_spmm_f32: null B");
    return dense_run<float>(true, *A, B, nullptr, C, k, sc, workspace, workspace_bytes, st);
}

int tg_spmm_f64(const tg_csr* A, const double* B, double* C, int64_t k, const tg_sched* s, void* workspace,
                size_t workspace_bytes, tg_stream_t stream) {
    TG_PRELUDE("tg_spmm_f64");
    if (A->rows > 0 && !C) return set_error(TG_EINVAL, "tg_spmm_f64: null C");
    if (A->nnz > 0 && !B) return set_error(TG_EINVAL, "tg_spmm_f64: null B");
    return dense_run<double>(true, *A, B, nullptr, C, k, sc, workspace, workspace_bytes, st);
}

int tg_sddmm_f32(const tg_csr* A, const float* U, const float* V, float* out, int64_t k, const tg_sched* s,
                 void* workspace, size_t workspace_bytes, tg_stream_t stream) {
    TG_PRELUDE("tg_sddmm_f32");
    if (A->nnz > 0 && (!U || !V || !out)) return set_error(TG_EINVAL, "tg_sddmm_f32: null U/V/out");
    return dense_run<float>(false, *A, V, U, out, k, sc, workspace, workspace_bytes, st);
}

int tg_sddmm_f64(const tg_csr* A, const double* U, const double* V, double* out, int64_t k, const tg_sched* s,
                 void* workspace, size_t workspace_bytes, tg_stream_t stream) {
    TG_PRELUDE("tg_sddmm_f64");
    if (A->nnz > 0 && (!U || !V || !out)) return set_error(TG_EINVAL, "tg_sddmm_f64: null U/V/out");
    return dense_run<double>(false, *A, V, U, out, k, sc, workspace, workspace_bytes, st);
}

int tg_axpy_f64(const double* x, const double* w, double* z, double alpha, double beta, int64_t n,
                const tg_sched* s, tg_stream_t stream) {
    tg_sched sc;
    int rc = resolve(s, &sc);
    if (rc != TG_OK) return rc;
    if (n < 0) return set_error(TG_EINVAL, "tg_axpy_f64: negative n");
    if (n > 0 && (!x || !w || !z)) return set_error(TG_EINVAL, "tg_axpy_f64: null x/w/z");
    const int64_t n_eff = (sc.flags & TG_FLAG_INJECT_BUG) && n > 0 ? n - 1 : n;
    return axpy_run<double>(x, w, z, alpha, beta, n_eff, sc.block_size, static_cast<cudaStream_t>(stream));
}

int tg_axpy_f32(const float* x, const float* w, float* z, float alpha, float beta, int64_t n, const tg_sched* s,
                tg_stream_t stream) {
    tg_sched sc;
    int rc = resolve(s, &sc);
    if (rc != TG_OK) return rc;
    if (n < 0) return set_error(TG_EINVAL, "tg_axpy_f32: negative n");
    if (n > 0 && (!x || !w || !z)) return set_error(TG_EINVAL, "tg_axpy_f32: null x/w/z");
    const int64_t n_eff = (sc.flags & TG_FLAG_INJECT_BUG) && n > 0 ? n - 1 : n;
    return axpy_run<float>(x, w, z, alpha, beta, n_eff, sc.block_size, static_cast<cudaStream_t>(stream));
}

size_t tg_power_workspace_bytes(int64_t nnz, const tg_sched* s) {
    tg_sched r;
    if (resolve(s, &r) != TG_OK) return 0;
    return power_ws_bytes(nnz, r);
}

int tg_power_step_f64(const tg_csr* A, const double* x, int32_t nparts, int64_t stride, double* y,
                      const tg_sched* s, void* workspace, size_t workspace_bytes, tg_stream_t stream) {
    TG_PRELUDE("tg_power_step_f64");
    if (!x || (A->rows > 0 && !y)) return set_error(TG_EINVAL, "tg_power_step_f64: null x/y");
    return power_step_run(*A, x, nparts, stride, y, sc, workspace, workspace_bytes, st);
}

int tg_shard_norm2_f64(double* shard, int64_t rows, int64_t stride, void* workspace, size_t workspace_bytes,
                       tg_stream_t stream) {
    if (!shard || rows < 0 || stride < rows + 1)
        return set_error(TG_EINVAL, "tg_shard_norm2_f64: bad shard (rows=%lld stride=%lld)", (long long)rows,
                         (long long)stride);
    return shard_norm2_run(shard, rows, stride, workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
}

int tg_power_finalize_f64(const double* x, int32_t nparts, int64_t stride, int32_t part, int64_t rows,
                          double* x_out, double* lambda_out, tg_stream_t stream) {
    if (!x || (rows > 0 && !x_out) || nparts < 1 || part < 0 || part >= nparts || stride < rows + 1)
        return set_error(TG_EINVAL, "tg_power_finalize_f64: bad arguments");
    return power_finalize_run(x, nparts, stride, part, rows, x_out, lambda_out, static_cast<cudaStream_t>(stream));
}

int tg_power_step_p2p_f64(const tg_csr* A, const double* x, int32_t nparts, int32_t rank, int64_t stride,
                          double* const* y_peers, uint64_t* const* flag_peers, uint64_t epoch, const tg_sched* s,
                          void* workspace, size_t workspace_bytes, tg_stream_t stream) {
    TG_PRELUDE("tg_power_step_p2p_f64");
    if (!x || !y_peers || !flag_peers) return set_error(TG_EINVAL, "tg_power_step_p2p_f64: null pointer");
    return power_step_p2p_run(*A, x, nparts, rank, stride, y_peers,
                              reinterpret_cast<unsigned long long* const*>(flag_peers), epoch, sc, workspace,
                              workspace_bytes, st);
}

int tg_power_error(const void* workspace, uint32_t* err, tg_stream_t stream) {
    if (!workspace || !err) return set_error(TG_EINVAL, "tg_power_error: null argument");
    const char* w = static_cast<const char*>(workspace) + power_err_offset();
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    int rc = check_cuda(cudaMemcpyAsync(err, w, sizeof(uint32_t), cudaMemcpyDeviceToHost, st), "cudaMemcpyAsync");
    if (rc != TG_OK) return rc;
    return check_cuda(cudaStreamSynchronize(st), "cudaStreamSynchronize");
}

int tg_power_step_ce_f64(const tg_csr* A, const double* x, int32_t nparts, int32_t rank, int64_t stride,
                         double* const* y_peers, uint64_t* const* flag_peers, uint64_t epoch, int32_t nchunks,
                         const tg_sched* s, void* workspace, size_t workspace_bytes, tg_stream_t stream) {
    TG_PRELUDE("tg_power_step_ce_f64");
    if (!x || !y_peers || !flag_peers) return set_error(TG_EINVAL, "tg_power_step_ce_f64: null pointer");
    return power_step_ce_run(*A, x, nparts, rank, stride, y_peers, reinterpret_cast<unsigned long long* const*>(flag_peers),
                             epoch, nchunks, sc, workspace, workspace_bytes, st);
}

int tg_power_clear_error(void* workspace, tg_stream_t stream) {
    if (!workspace) return set_error(TG_EINVAL, "tg_power_clear_error: null workspace");
    char* w = static_cast<char*>(workspace) + power_err_offset();
    return check_cuda(cudaMemsetAsync(w, 0, sizeof(uint32_t), static_cast<cudaStream_t>(stream)), "cudaMemsetAsync");
}

int tg_p2p_wait(const uint64_t* flag_local, int32_t nparts, uint64_t epoch, void* workspace, size_t workspace_bytes,
                tg_stream_t stream) {
    return p2p_wait_run(reinterpret_cast<const unsigned long long*>(flag_local), nparts, epoch, workspace,
                        workspace_bytes, static_cast<cudaStream_t>(stream));
}

// ------------------------------------------------ peer buffers (multi-GPU exchange)
int tg_peer_buffer_alloc(size_t bytes, void** ptr) {
    if (!ptr || bytes == 0) return set_error(TG_EINVAL, "tg_peer_buffer_alloc: bad arguments");
    *ptr = nullptr;
    int rc = check_cuda(cudaMalloc(ptr, bytes), "cudaMalloc(peer buffer)");
    if (rc != TG_OK) return rc;
    rc = check_cuda(cudaMemset(*ptr, 0, bytes), "cudaMemset(peer buffer)");
    if (rc != TG_OK) {
        cudaFree(*ptr);
        *ptr = nullptr;
    }
    return rc;
}

int tg_peer_buffer_free(void* ptr) { return ptr ? check_cuda(cudaFree(ptr), "cudaFree(peer buffer)") : TG_OK; }

int tg_ipc_get_handle(const void* ptr, void* handle) {
    if (!ptr || !handle) return set_error(TG_EINVAL, "tg_ipc_get_handle: null argument");
    static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
    cudaIpcMemHandle_t h;
    int rc = check_cuda(cudaIpcGetMemHandle(&h, const_cast<void*>(ptr)), "cudaIpcGetMemHandle");
    if (rc == TG_OK) memcpy(handle, &h, sizeof(h));
    return rc;
}

int tg_ipc_open(const void* handle, void** ptr) {
    if (!handle || !ptr) return set_error(TG_EINVAL, "tg_ipc_open: null argument");
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    *ptr = nullptr;
    return check_cuda(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
}

int tg_ipc_close(void* ptr) { return ptr ? check_cuda(cudaIpcCloseMemHandle(ptr), "cudaIpcCloseMemHandle") : TG_OK; }

// ------------------------------------------------ reference-compatible launchers
static void finish_shim(int rc) {
    if (rc == TG_OK) rc = check_cuda(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
    t_last_status = rc;
    if (rc == TG_OK) t_msg[0] = '\0';
}

void launch_spmv(const int64_t* indptr, const int64_t* indices, const double* data, const double* x, double* y,
                 int64_t M, int64_t N, int64_t nnz) {
    std::lock_guard<std::mutex> shim_lock(g_shim_mu);
    tg_sched s;
    tg_get_schedule(&s);
    tg_csr A{M, N, nnz, indptr, indices, data};
    int rc = TG_OK;
    const size_t need = tg_spmv_workspace_bytes(M, nnz, &s);
    void* ws = shim_workspace(need, &rc);
    if (rc == TG_OK) rc = tg_spmv_f64(&A, x, y, &s, ws, need, nullptr);
    finish_shim(rc);
}

void launch_spmm(const int64_t* indptr, const int64_t* indices, const double* data, const double* B, double* C,
                 int64_t M, int64_t N, int64_t K, int64_t nnz) {
    std::lock_guard<std::mutex> shim_lock(g_shim_mu);
    tg_sched s;
    tg_get_schedule(&s);
    tg_csr A{M, N, nnz, indptr, indices, data};
    int rc = TG_OK;
    const size_t need = tg_spmm_workspace_bytes(M, nnz, K, &s);
    void* ws = shim_workspace(need, &rc);
    if (rc == TG_OK) rc = tg_spmm_f64(&A, B, C, K, &s, ws, need, nullptr);
    finish_shim(rc);
}

void launch_sddmm(const int64_t* indptr, const int64_t* indices, const double* data, const double* U,
                  const double* V, double* C, int64_t M, int64_t N, int64_t K, int64_t nnz) {
    std::lock_guard<std::mutex> shim_lock(g_shim_mu);
    tg_sched s;
    tg_get_schedule(&s);
    tg_csr A{M, N, nnz, indptr, indices, data};
    int rc = TG_OK;
    const size_t need = tg_sddmm_workspace_bytes(M, nnz, K, &s);
    void* ws = shim_workspace(need, &rc);
    if (rc == TG_OK) rc = tg_sddmm_f64(&A, U, V, C, K, &s, ws, need, nullptr);
    finish_shim(rc);
}

void launch_fused_spmv_axpy(const int64_t* indptr, const int64_t* indices, const double* data, const double* x,
                            const double* w, double* z, double alpha, double beta, int64_t M, int64_t N,
                            int64_t nnz) {
    std::lock_guard<std::mutex> shim_lock(g_shim_mu);
    tg_sched s;
    tg_get_schedule(&s);
    tg_csr A{M, N, nnz, indptr, indices, data};
    int rc = TG_OK;
    const size_t need = tg_spmv_workspace_bytes(M, nnz, &s);
    void* ws = shim_workspace(need, &rc);
    if (rc == TG_OK) rc = tg_fused_spmv_axpy_f64(&A, x, w, z, alpha, beta, &s, ws, need, nullptr);
    finish_shim(rc);
}

void launch_axpy(const double* x, const double* w, double* z, double alpha, double beta, int64_t M) {
    std::lock_guard<std::mutex> shim_lock(g_shim_mu);
    tg_sched s;
    tg_get_schedule(&s);
    finish_shim(tg_axpy_f64(x, w, z, alpha, beta, M, &s, nullptr));
}

}  // extern "C"
