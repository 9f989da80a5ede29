// CSR SpMV (and the fused SpMV+axpy epilogue) for sm_100a.
//
// Reference: the emitted `scalar_reduce` templates K1/K2 (tilegen/codegen.py:592-643),
// launch wrapper tilegen/codegen.py:764-799; math cpp/src/ref.cpp:6-15 (spmv) and
// :62-73 (fused_spmv_axpy).
//
// Two row mappings:
//  * rowwise  -- the reference schedule space made sound and fast: a CTA owns tiles of
//    T rows, TPR lanes cooperate on a row (segmented shuffle with the group's own lane
//    mask, so tails are well defined), each lane keeps U vector loads of V nonzeros in
//    flight, indices/values stream with an L2 evict_first policy and x is gathered with
//    evict_last.  Template parameters: TPR, U, V; runtime: T, B.
//  * merge    -- nnz-balanced chunks of S = B*I nonzeros per CTA.  The CTA computes
//    the chunk's products into shared memory (I coalesced loads and I gathers in flight
//    per thread), then sums each row's piece from shared memory: short pieces by one
//    thread, long ones by a warp.  A row crossing chunk boundaries gets one partial per
//    chunk; the last of its contributors to arrive (acq_rel atomic) adds them in chunk
//    order and writes the row, inside the same kernel.  Power-law rows of any length cost
//    the same per nonzero as short rows, and no CTA ever waits for another.  The
//    partition table (the plan) can be kept across calls on the same matrix.
#include <algorithm>

#include "tg_rowdot.cuh"
#include "tg_split.cuh"

namespace tg {

// ------------------------------------------------------------------ rowwise
template <typename T>
struct SpmvArgs {
    const int64_t* indptr;
    const int64_t* indices;
    const T* data;
    const T* x;
    T* y;
    int64_t rows;
    int64_t nnz;
    int64_t rows_per_tile;  // rowwise: rows a CTA owns per tile (>= its lane groups)
    int64_t row_limit;      // rows >= row_limit are not written (injected-bug self test)
    // merge split
    const int64_t* own_first;
    int* cnt;
    T* head;
    T* tail;
    uint32_t* err;
};

template <typename T, int TPR, int U, int V, bool AXPY>
__global__ void __launch_bounds__(512) spmv_rowwise_kernel(SpmvArgs<T> a, Epi<T, AXPY> epi) {
    const uint64_t ps = policy_evict_first();
    const uint64_t pg = policy_evict_last();
    const int lane = threadIdx.x % TPR;
    const int group = threadIdx.x / TPR;
    const int groups = blockDim.x / TPR;
    unsigned mask = kFull;
    if constexpr (TPR < 32) mask = ((1u << TPR) - 1u) << ((threadIdx.x % 32) / TPR * TPR);
    for (int64_t base = (int64_t)blockIdx.x * a.rows_per_tile; base < a.rows;
         base += (int64_t)gridDim.x * a.rows_per_tile) {
        const int64_t end = min(base + a.rows_per_tile, a.rows);
        for (int64_t i = base + group; i < end; i += groups) {
            const int64_t p = a.indptr[i];
            const int64_t pe = a.indptr[i + 1];
            T acc = row_dot<T, TPR, U, V>(a.indices, a.data, a.x, p, pe, lane, ps, pg);
            if constexpr (TPR > 1) acc = group_sum<TPR>(acc, mask);
            if (lane == 0 && i < a.row_limit) a.y[i] = epi(acc, i);
        }
    }
}

// ------------------------------------------------------------------ merge
constexpr int kMergeI = 7;  // nonzeros per thread

// Rows whose piece of a chunk is at most this long are summed by one thread; longer
// pieces by a whole warp.
constexpr int kShortPiece = 16;

// Arrival count at which every contributor of a split row has published its partial:
// the owner adds kArriveAll - (number of later chunks the row covers), each later chunk
// adds 1, so the sum reaches kArriveAll exactly once, at the last arrival.
constexpr int kArriveAll = 1 << 30;

__device__ __forceinline__ int atomic_add_acq_rel(int* p, int v) {
    int old;
    asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}

// A row whose nonzeros cross chunk boundaries spans chunks ca..cb: its owner ca publishes
// tail[ca], every later chunk c' publishes head[c'], and each then arrives on cnt[cb]
// (one split row ends in a chunk, so cb names the row).  The arrival is an acq_rel
// atomic: it releases this contributor's partial and, for the last arrival, acquires
// every other one.  The last arrival adds tail[ca] + head[ca+1] + ... + head[cb] in that
// fixed order (the result does not depend on which contributor came last), writes the
// row and resets cnt[cb] for the next call.
template <typename T, bool AXPY>
__device__ __forceinline__ void merge_arrive(const SpmvArgs<T>& a, const Epi<T, AXPY>& epi, int64_t r, int64_t ca,
                                             int64_t cb, int64_t c, int64_t S, T v) {
    (c == ca ? a.tail : a.head)[c] = v;
    const int add = (c == ca) ? kArriveAll - (int)(cb - ca) : 1;
    const int old = atomic_add_acq_rel(&a.cnt[cb], add);
    if (old + add != kArriveAll) return;
    if (ca < 0) ca = a.indptr[r] / S;  // a head contributor came last: find the owner
    Sum<T> sum;
    sum.add(ld_cg(&a.tail[ca]));
    add_partials(sum, a.head + ca + 1, cb - ca, 1);
    if (r < a.row_limit) a.y[r] = epi(sum.get(), r);
    a.cnt[cb] = 0;
}

// Chunk c holds nonzeros [c*S, c*S + S) with S = B*I.  Its CTA
//  1. issues the chunk's coalesced index/value loads (I per thread) and, at the same
//     time, the loads of its rows' offsets (partition table, then the indptr slice of
//     the rows that start in the chunk), then the I gathers of x, and stores the S
//     products in shared memory;
//  2. sums every row piece from shared memory in index order: short pieces by one
//     thread, long pieces by a warp (strided partial sums, then a fixed shuffle tree).
// A row that lies inside the chunk is written to y.  The piece of a row that started in
// an earlier chunk (the chunk's head) and the piece of the chunk's last row when it
// continues into later chunks (its tail) are combined with the row's other pieces by
// merge_arrive, in this kernel: no fix-up launch.  On a planning call the partition
// kernel runs just before (programmatic launch) and the table is read after pdl_wait;
// with the plan reused there is no kernel before it and pdl_wait returns at once.
template <typename T, bool AXPY, int B>
__global__ void __launch_bounds__(B) spmv_merge_kernel(SpmvArgs<T> a, Epi<T, AXPY> epi) {
    constexpr int I = kMergeI;
    constexpr int S = B * I;
    constexpr int RCAP = S + 32;
    constexpr int NW = B / kWarp;
    __shared__ T s_prod[S];
    __shared__ int64_t s_off[RCAP];
    __shared__ int s_long[S / kShortPiece + 2];
    __shared__ int s_nlong;

    const int tid = threadIdx.x;
    const int64_t c = blockIdx.x;
    const int64_t cs = c * S;
    const int64_t ce = min(cs + (int64_t)S, a.nnz);
    const int n_items = (int)(ce - cs);
    const uint64_t ps = policy_evict_first();
    const uint64_t pg = policy_evict_last();

    // 1. CSR stream loads, then the row offsets (independent of them), then the gathers
    int64_t col[I];
    T val[I];
#pragma unroll
    for (int k = 0; k < I; ++k) {
        const int q = tid + k * B;
        col[k] = 0;
        val[k] = T(0);
        if (q < n_items) {
            col[k] = ld_stream(a.indices + cs + q, ps);
            val[k] = ld_stream(a.data + cs + q, ps);
        }
    }
    pdl_wait();  // planning call: the partition kernel before this one wrote the table
    const int64_t of0 = a.own_first[c];
    const int64_t of1 = a.own_first[c + 1];
    const int64_t n_off = of1 - of0 + 1;
    const bool off_smem = n_off <= RCAP;
    if (off_smem)
        for (int64_t j = tid; j < n_off; j += B) s_off[j] = a.indptr[of0 + j];
    if (tid == 0) s_nlong = 0;
#pragma unroll
    for (int k = 0; k < I; ++k) {
        const int q = tid + k * B;
        if (q < n_items) s_prod[q] = val[k] * ld_gather(a.x + col[k], pg);
    }
    __syncthreads();
    const int64_t* off = off_smem ? s_off : (a.indptr + of0);

    // 2. pieces: task 0 is the head (the row before of0, continuing into the chunk), task
    //    1 + j is row of0 + j.  Piece [lo, hi) in chunk coordinates.
    const int64_t ntask = n_off;  // head + (of1 - of0) rows
    auto piece = [&](int64_t t, int& lo, int& hi) {
        if (t == 0) {
            lo = 0;
            hi = (int)(min(off[0], ce) - cs);
        } else {
            lo = (int)(off[t - 1] - cs);
            hi = (int)(min(off[t], ce) - cs);
        }
    };
    auto finish = [&](int64_t t, T v) {
        if (t == 0) {  // head: row of0 - 1 ends in chunk (off[0] - 1) / S, owner unknown here
            merge_arrive<T, AXPY>(a, epi, of0 - 1, -1, (off[0] - 1) / S, c, S, v);
        } else {
            const int64_t r = of0 + t - 1;
            if (off[t] <= ce) {
                if (r < a.row_limit) a.y[r] = epi(v, r);
            } else {  // the chunk's last row continues past the chunk
                merge_arrive<T, AXPY>(a, epi, r, c, (off[t] - 1) / S, c, S, v);
            }
        }
    };
    for (int64_t t = tid; t < ntask; t += B) {
        int lo, hi;
        piece(t, lo, hi);
        if (t == 0 && hi <= 0) continue;  // no head
        if (hi - lo > kShortPiece) {
            s_long[atomicAdd(&s_nlong, 1)] = (int)t;
            continue;
        }
        Sum<T> sum;
        for (int q = lo; q < hi; ++q) sum.add(s_prod[q]);
        finish(t, sum.get());
    }
    __syncthreads();
    const int nlong = s_nlong;
    const int warp = tid / kWarp, lane = tid % kWarp;
    for (int i = warp; i < nlong; i += NW) {
        const int64_t t = s_long[i];
        int lo, hi;
        piece(t, lo, hi);
        Sum<T> sum;
        for (int q = lo + lane; q < hi; q += kWarp) sum.add(s_prod[q]);
        const T v = group_sum<kWarp>(sum.get(), kFull);
        if (lane == 0) finish(t, v);
    }
}

// ------------------------------------------------------------------ small kernels
template <typename T, bool AXPY>
__global__ void fill_rows_kernel(T* y, int64_t rows, int64_t row_limit, Epi<T, AXPY> epi) {
    for (int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; r < rows && r < row_limit;
         r += (int64_t)gridDim.x * blockDim.x)
        y[r] = epi(T(0), r);
}

template <typename T>
__global__ void axpy_kernel(const T* __restrict__ x, const T* __restrict__ w, T* __restrict__ z, T alpha, T beta,
                            int64_t n) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        z[i] = alpha * x[i] + beta * w[i];
}

// ------------------------------------------------------------------ host side
namespace {

template <typename T, bool AXPY, int TPR, int U, int V>
void launch_rowwise(const SpmvArgs<T>& a, const Epi<T, AXPY>& epi, int64_t blocks, int threads, cudaStream_t st) {
    spmv_rowwise_kernel<T, TPR, U, V, AXPY><<<(unsigned)blocks, threads, 0, st>>>(a, epi);
}

template <typename T, bool AXPY, int TPR, int U>
bool dispatch_v(int v, const SpmvArgs<T>& a, const Epi<T, AXPY>& e, int64_t bl, int th, cudaStream_t st) {
    switch (v) {
        case 1: launch_rowwise<T, AXPY, TPR, U, 1>(a, e, bl, th, st); return true;
        case 2: launch_rowwise<T, AXPY, TPR, U, 2>(a, e, bl, th, st); return true;
        case 4: launch_rowwise<T, AXPY, TPR, U, 4>(a, e, bl, th, st); return true;
    }
    return false;
}

template <typename T, bool AXPY, int TPR>
bool dispatch_u(int u, int v, const SpmvArgs<T>& a, const Epi<T, AXPY>& e, int64_t bl, int th, cudaStream_t st) {
    switch (u) {
        case 1: return dispatch_v<T, AXPY, TPR, 1>(v, a, e, bl, th, st);
        case 2: return dispatch_v<T, AXPY, TPR, 2>(v, a, e, bl, th, st);
        case 4: return dispatch_v<T, AXPY, TPR, 4>(v, a, e, bl, th, st);
        case 8: return dispatch_v<T, AXPY, TPR, 8>(v, a, e, bl, th, st);
    }
    return false;
}

template <typename T, bool AXPY>
bool dispatch_rowwise(int tpr, int u, int v, const SpmvArgs<T>& a, const Epi<T, AXPY>& e, int64_t bl, int th,
                      cudaStream_t st) {
    switch (tpr) {
        case 1: return dispatch_u<T, AXPY, 1>(u, v, a, e, bl, th, st);
        case 2: return dispatch_u<T, AXPY, 2>(u, v, a, e, bl, th, st);
        case 4: return dispatch_u<T, AXPY, 4>(u, v, a, e, bl, th, st);
        case 8: return dispatch_u<T, AXPY, 8>(u, v, a, e, bl, th, st);
        case 16: return dispatch_u<T, AXPY, 16>(u, v, a, e, bl, th, st);
        case 32: return dispatch_u<T, AXPY, 32>(u, v, a, e, bl, th, st);
    }
    return false;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

int64_t merge_chunk_nnz(int block) { return (int64_t)block * kMergeI; }

int merge_block(const tg_sched& s) { return s.block_size == 128 ? 128 : 256; }

// stream split (tg_stream.cu)
enum StreamModeFwd { kStreamPlain = 0, kStreamAxpy = 1 };
template <typename T, int MODE>
int stream_run(const tg_csr& A, const T* x, T* y, const T* w, T alpha, T beta, int nparts, int64_t stride,
               const tg_sched& s, void* ws, size_t ws_bytes, cudaStream_t st);
size_t stream_ws_bytes(int64_t nnz, const tg_sched& s, size_t elem);

static bool stream_ok(const tg_csr& A) {
    return A.nnz > 0 && ((reinterpret_cast<uintptr_t>(A.indices) | reinterpret_cast<uintptr_t>(A.data) |
                          reinterpret_cast<uintptr_t>(A.indptr)) & 15u) == 0;
}

size_t spmv_ws_bytes(int64_t rows, int64_t nnz, const tg_sched& s, size_t elem) {
    (void)rows;
    if (s.split == TG_SPLIT_STREAM && nnz > 0)
        return std::max(stream_ws_bytes(nnz, s, elem),
                        split_ws_bytes(ceil_div(nnz, merge_chunk_nnz(merge_block(s))), 1, elem));
    if ((s.split != TG_SPLIT_MERGE && s.split != TG_SPLIT_BLOCK) || nnz <= 0) return 0;
    const int64_t S = merge_chunk_nnz(merge_block(s));
    return split_ws_bytes(ceil_div(nnz, S), 1, elem);
}

template <typename T, bool AXPY>
int spmv_run(const tg_csr& A, const T* x, T* y, const Epi<T, AXPY>& epi, const tg_sched& s, void* ws,
             size_t ws_bytes, cudaStream_t st) {
    const int64_t row_limit = (s.flags & TG_FLAG_INJECT_BUG) ? A.rows - 1 : A.rows;
    if (A.rows == 0) return TG_OK;
    SpmvArgs<T> a{};
    a.indptr = A.indptr;
    a.indices = A.indices;
    a.data = static_cast<const T*>(A.data);
    a.x = x;
    a.y = y;
    a.rows = A.rows;
    a.nnz = A.nnz;
    a.row_limit = row_limit;
    if (A.nnz == 0) {
        int64_t blocks = std::min<int64_t>(ceil_div(A.rows, 256), 148 * 8);
        fill_rows_kernel<T, AXPY><<<(unsigned)blocks, 256, 0, st>>>(y, A.rows, row_limit, epi);
        return check_launch("fill_rows_kernel");
    }
    if (s.split == TG_SPLIT_STREAM && stream_ok(A)) {
        if constexpr (AXPY) {
            return stream_run<T, kStreamAxpy>(A, x, y, epi.w, epi.alpha, epi.beta, 1, 0, s, ws, ws_bytes, st);
        } else {
            return stream_run<T, kStreamPlain>(A, x, y, nullptr, T(0), T(0), 1, 0, s, ws, ws_bytes, st);
        }
    }
    if (s.split == TG_SPLIT_MERGE || s.split == TG_SPLIT_STREAM || s.split == TG_SPLIT_BLOCK) {
        // stream needs 16-byte aligned operands; the merge split handles any alignment
        // (the block split is an SpMM mapping: SpMV takes the merge split for it)
        const int B = merge_block(s);
        const int64_t S = merge_chunk_nnz(B);
        const int64_t nchunks = ceil_div(A.nnz, S);
        const size_t need = split_ws_bytes(nchunks, 1, sizeof(T));
        if (ws == nullptr || ws_bytes < need)
            return set_error(TG_ENOMEM, "spmv merge split needs %zu workspace bytes, got %zu", need, ws_bytes);
        if (nchunks > 0x7fffffff) return set_error(TG_EINVAL, "too many chunks (%lld)", (long long)nchunks);
        SplitWs w = split_ws_carve(ws, nchunks, 1, sizeof(T));
        // The plan (partition table, zeroed arrival counters) depends only on A's row
        // offsets and the chunk size.  TG_FLAG_REUSE_PLAN: the workspace already holds it
        // from an earlier call on the same A with the same schedule; every call leaves
        // the counters at zero again.
        const bool reuse = (s.flags & TG_FLAG_REUSE_PLAN) != 0;
        if (!reuse) {
            int rc = launch_partition(A.indptr, A.rows, A.nnz, S, w, st);
            if (rc != TG_OK) return rc;
        }
        a.own_first = w.own_first;
        a.cnt = w.cnt;
        a.head = static_cast<T*>(w.head);
        a.tail = static_cast<T*>(w.tail);
        a.err = w.err;
        // planning call: programmatic launch, so the chunk loads overlap the partition
        cudaLaunchConfig_t cfg = {};
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.gridDim = dim3((unsigned)nchunks);
        cfg.blockDim = dim3((unsigned)B);
        cfg.dynamicSmemBytes = 0;
        cfg.stream = st;
        cfg.attrs = reuse ? nullptr : attr;
        cfg.numAttrs = reuse ? 0 : 1;
        cudaError_t e = B == 128 ? cudaLaunchKernelEx(&cfg, spmv_merge_kernel<T, AXPY, 128>, a, epi)
                                 : cudaLaunchKernelEx(&cfg, spmv_merge_kernel<T, AXPY, 256>, a, epi);
        if (e != cudaSuccess) return check_cuda(e, "spmv_merge_kernel launch");
        return check_launch("spmv_merge_kernel");
    }
    // rowwise
    const int tpr = s.threads_per_row;
    int v = s.vector_width;
    if (!(aligned16(A.indices) && aligned16(A.data))) v = 1;
    const int threads = s.block_size;
    const int64_t groups = threads / tpr;
    a.rows_per_tile = std::max<int64_t>(s.tile, groups);
    int64_t blocks = ceil_div(A.rows, a.rows_per_tile);
    if (blocks > (1 << 20)) blocks = 1 << 20;
    if (!dispatch_rowwise<T, AXPY>(tpr, s.unroll, v, a, epi, blocks, threads, st))
        return set_error(TG_EUNSUPPORTED, "no rowwise SpMV instance for TPR=%d U=%d V=%d", tpr, s.unroll, v);
    return check_launch("spmv_rowwise_kernel");
}

template int spmv_run<double, false>(const tg_csr&, const double*, double*, const Epi<double, false>&,
                                     const tg_sched&, void*, size_t, cudaStream_t);
template int spmv_run<double, true>(const tg_csr&, const double*, double*, const Epi<double, true>&,
                                    const tg_sched&, void*, size_t, cudaStream_t);
template int spmv_run<float, false>(const tg_csr&, const float*, float*, const Epi<float, false>&, const tg_sched&,
                                    void*, size_t, cudaStream_t);
template int spmv_run<float, true>(const tg_csr&, const float*, float*, const Epi<float, true>&, const tg_sched&,
                                   void*, size_t, cudaStream_t);

template <typename T>
int axpy_run(const T* x, const T* w, T* z, T alpha, T beta, int64_t n, int block, cudaStream_t st) {
    if (n == 0) return TG_OK;
    int64_t blocks = std::min<int64_t>(ceil_div(n, block), 148 * 16);
    axpy_kernel<T><<<(unsigned)blocks, block, 0, st>>>(x, w, z, alpha, beta, n);
    return check_launch("axpy_kernel");
}
template int axpy_run<double>(const double*, const double*, double*, double, double, int64_t, int, cudaStream_t);
template int axpy_run<float>(const float*, const float*, float*, float, float, int64_t, int, cudaStream_t);

}  // namespace tg
