// tg_spmv_f64_noalloc: the merge-split SpMV for callers that cannot allocate device
// memory.
//
// Some callers can hand this library only their inputs and outputs: a plugin host that
// owns every byte of the GPU through its own pool and forbids side allocations, or code
// on a latency-critical path where cudaMalloc's implicit device synchronisation (and its
// chance of failing under memory pressure) is not acceptable.  The regular tg_spmv_f64
// needs a caller-provided workspace for the merge split; this entry point instead keeps
// that scratch in a fixed array in the library's device memory.
//
// * The scratch is g_noalloc_scratch below: kNoAllocScratchBytes (1 MiB) per GPU, present
//   on every GPU that loads the library, for as long as the process runs.
// * Host code cannot use the array's name as a device address.  The first call on a
//   device looks the address up with cudaGetSymbolAddress while that device is current,
//   checks the result and caches it; that first call should therefore come before any
//   stream capture on the device.  The cached address belongs to the device's current
//   context: after cudaDeviceReset (or anything else that destroys the primary context
//   and reloads the module) it is stale, so such a program must not call this entry
//   point again in the same process.
// * Calls that need more scratch than the array holds are rejected with TG_EINVAL and a
//   message giving the limit; nothing here calls cudaMalloc, cudaFree or any allocating
//   routine.
// * Every call shares the one array.  Whatever must start at zero (the split-row
//   counters and the error word) is cleared by the partition pass at the start of each
//   call; the rest is written before it is read.  Calls whose kernels overlap on the GPU
//   (different streams, no ordering between them) race on the array: serialise them.
#include <mutex>

#include "tg_split.cuh"

namespace tg {
template <typename T, bool AXPY>
int spmv_run(const tg_csr& A, const T* x, T* y, const Epi<T, AXPY>& epi, const tg_sched& s, void* ws,
             size_t ws_bytes, cudaStream_t st);
int64_t merge_chunk_nnz(int block);
int merge_block(const tg_sched& s);
int resolve_schedule(const tg_sched* in, tg_sched* out);
}  // namespace tg

using namespace tg;

static constexpr size_t kNoAllocScratchBytes = size_t(1) << 20;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

namespace {

constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
void* g_noalloc_ptr[kMaxDevices] = {};

// Device address of g_noalloc_scratch on the current device (looked up once per device).
int scratch_address(void** out) {
    int dev = 0;
    int rc = check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
    if (rc != TG_OK) return rc;
    if (dev < 0 || dev >= kMaxDevices) return set_error(TG_EUNSUPPORTED, "device %d out of range", dev);
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (!g_noalloc_ptr[dev]) {
        void* p = nullptr;
        rc = check_cuda(cudaGetSymbolAddress(&p, g_noalloc_scratch), "cudaGetSymbolAddress(g_noalloc_scratch)");
        if (rc != TG_OK) return rc;
        g_noalloc_ptr[dev] = p;
    }
    *out = g_noalloc_ptr[dev];
    return TG_OK;
}

}  // namespace

extern "C" int tg_spmv_f64_noalloc(const tg_csr* A, const double* x, double* y, const tg_sched* s,
                                   tg_stream_t stream) {
    if (!A) return set_error(TG_EINVAL, "tg_spmv_f64_noalloc: null CSR descriptor");
    if (A->rows < 0 || A->cols < 0 || A->nnz < 0)
        return set_error(TG_EINVAL, "tg_spmv_f64_noalloc: negative size");
    if (!A->indptr || (A->nnz > 0 && (!A->indices || !A->data || !x)) || (A->rows > 0 && !y))
        return set_error(TG_EINVAL, "tg_spmv_f64_noalloc: null pointer argument");
    // the schedule tg_spmv_f64 would use (NULL: the process schedule), with the merge split
    tg_sched sc;
    int rc = resolve_schedule(s, &sc);
    if (rc != TG_OK) return rc;
    sc.split = TG_SPLIT_MERGE;
    if (sc.flags & (TG_FLAG_BOUNDS_CHECK | TG_FLAG_REUSE_PLAN))
        return set_error(TG_EINVAL, "tg_spmv_f64_noalloc: bounds checking and plan reuse are not available here");
    const int64_t S = merge_chunk_nnz(merge_block(sc));
    const int64_t nchunks = A->nnz > 0 ? ceil_div(A->nnz, S) : 0;
    const size_t need = A->nnz > 0 ? split_ws_bytes(nchunks, 1, sizeof(double)) : 0;
    if (need > kNoAllocScratchBytes) {
        // largest chunk count whose scratch fits, for the message
        int64_t lo = 0, hi = nchunks;
        while (lo < hi) {
            const int64_t mid = (lo + hi + 1) / 2;
            if (split_ws_bytes(mid, 1, sizeof(double)) <= kNoAllocScratchBytes)
                lo = mid;
            else
                hi = mid - 1;
        }
        return set_error(TG_EINVAL,
                         "tg_spmv_f64_noalloc: nnz=%lld needs %zu bytes of scratch, more than the fixed %zu "
                         "(at most %lld nonzeros with block_size %d); use tg_spmv_f64 with a workspace",
                         (long long)A->nnz, need, kNoAllocScratchBytes, (long long)(lo * S), merge_block(sc));
    }
    void* ws = nullptr;
    rc = scratch_address(&ws);
    if (rc != TG_OK) return rc;
    return spmv_run<double, false>(*A, x, y, Epi<double, false>{nullptr, 0.0, 0.0}, sc, ws, kNoAllocScratchBytes,
                                   static_cast<cudaStream_t>(stream));
}
