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
//  * merge    -- nnz-balanced chunks of S = B*I nonzeros per CTA.  The chunk's indices
//    and values are staged into shared memory by one TMA bulk copy (cp.async.bulk +
//    mbarrier), row offsets by coalesced loads; each thread multiplies I consecutive
//    nonzeros (all gathers in flight at once) and then walks them against the row
//    offsets (merge of row ends and nonzero positions).  Rows crossing thread
//    boundaries are summed by their owner thread; rows crossing chunk boundaries use
//    the deterministic last-arriver protocol of tg_split.cuh.  Power-law rows of any
//    length cost the same per nonzero as short rows.
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
    int use_bulk;
};

template <typename T, int TPR, int U, int V, bool AXPY>
__global__ void __launch_bounds__(1024) spmv_rowwise_kernel(SpmvArgs<T> a, Epi<T, AXPY> epi) {
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
constexpr int kMergeI = 7;  // nonzeros per thread; odd => conflict-free 8-byte smem reads

template <typename T, bool AXPY, int B>
__global__ void __launch_bounds__(B) spmv_merge_kernel(SpmvArgs<T> a, Epi<T, AXPY> epi) {
    constexpr int I = kMergeI;
    constexpr int S = B * I;
    constexpr int RCAP = S + 32;
    __shared__ alignas(128) unsigned char s_raw[S * 8 + S * sizeof(T)];
    __shared__ alignas(16) int64_t s_off[RCAP];
    __shared__ alignas(8) uint64_t s_bar;
    int64_t* s_idx = reinterpret_cast<int64_t*>(s_raw);
    T* s_val = reinterpret_cast<T*>(s_raw + S * 8);

    const int tid = threadIdx.x;
    const int64_t c = blockIdx.x;
    const int64_t cs = c * S;
    const int64_t ce = min(cs + (int64_t)S, a.nnz);
    const int64_t n_items = ce - cs;
    const uint64_t ps = policy_evict_first();
    const uint64_t pg = policy_evict_last();

    // 1. stage this chunk's indices and values: one TMA bulk copy each (16-byte granules),
    //    the few trailing elements with plain loads.
    constexpr int64_t kGran = (sizeof(T) == 4) ? 4 : 2;
    const int64_t n_bulk = a.use_bulk ? (n_items / kGran) * kGran : 0;
    if (tid == 0) {
        mbar_init(&s_bar, 1);
        fence_mbar_init();
        if (n_bulk > 0) {
            const uint32_t bi = (uint32_t)(n_bulk * 8);
            const uint32_t bv = (uint32_t)(n_bulk * sizeof(T));
            mbar_arrive_expect_tx(&s_bar, bi + bv);
            bulk_g2s(s_idx, a.indices + cs, bi, &s_bar, ps);
            bulk_g2s(s_val, a.data + cs, bv, &s_bar, ps);
        } else {
            asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(&s_bar)) : "memory");
        }
    }
    for (int64_t k = n_bulk + tid; k < n_items; k += B) {
        s_idx[k] = ld_stream(a.indices + cs + k, ps);
        s_val[k] = ld_stream(a.data + cs + k, ps);
    }

    // 2. row offsets touching the chunk: indptr[r_lo .. r_hi+1]
    const int64_t of0 = a.own_first[c];
    const int64_t of1 = a.own_first[c + 1];
    const int64_t r_lo = of0 > 0 ? of0 - 1 : 0;
    const int64_t r_hi = of1 - 1;
    const int64_t n_off = r_hi + 2 - r_lo;
    const bool off_smem = n_off <= RCAP;
    if (off_smem)
        for (int64_t j = tid; j < n_off; j += B) s_off[j] = a.indptr[r_lo + j];
    __syncthreads();
    if (!mbar_wait(&s_bar, 0)) {
        if (tid == 0) atomicOr(a.err, 1u);
        return;
    }
    const int64_t* off = off_smem ? s_off : (a.indptr + r_lo);

    // 3. products of this thread's I nonzeros, then the merge walk
    const int64_t qa = cs + (int64_t)tid * I;
    const int64_t qb = min(qa + (int64_t)I, ce);
    int64_t h_row = -1, t_row = -1;
    T h_val = T(0), t_val = T(0);
    if (qa < qb) {
        T prod[I];
#pragma unroll
        for (int k = 0; k < I; ++k) {
            const int64_t q = qa + k;
            prod[k] = T(0);
            if (q < qb) {
                const int64_t li = q - cs;
                prod[k] = s_val[li] * ld_gather(a.x + s_idx[li], pg);
            }
        }
        // first row of the walk: empty rows starting exactly at qa, else the row containing qa
        int64_t lo = 0, hi = n_off;
        while (lo < hi) {
            const int64_t mid = (lo + hi) >> 1;
            if (off[mid] < qa)
                lo = mid + 1;
            else
                hi = mid;
        }
        int64_t j = (lo < n_off && off[lo] == qa) ? lo : lo - 1;
        const bool head = off[j] < qa;
        bool first = true;
        Sum<T> acc;
        int64_t nxt = off[j + 1];
#pragma unroll
        for (int k = 0; k < I; ++k) {
            const int64_t q = qa + k;
            if (q < qb) {
                while (nxt <= q) {
                    const int64_t r = r_lo + j;
                    if (first && head) {
                        h_row = r;
                        h_val = acc.get();
                    } else if (r < a.row_limit) {
                        a.y[r] = epi(acc.get(), r);
                    }
                    first = false;
                    acc = Sum<T>();
                    ++j;
                    nxt = off[j + 1];
                }
                acc.add(prod[k]);
            }
        }
        const int64_t r = r_lo + j;
        if (nxt == qb) {
            if (first && head) {
                h_row = r;
                h_val = acc.get();
            } else if (r < a.row_limit) {
                a.y[r] = epi(acc.get(), r);
            }
            if (qb == a.nnz)  // trailing empty rows (start == end == nnz)
                for (int64_t rr = r + 1; rr < a.rows && rr < a.row_limit; ++rr) a.y[rr] = epi(T(0), rr);
        } else if (first && head) {
            h_row = r;  // the whole range lies inside one row that started earlier
            h_val = acc.get();
        } else {
            t_row = r;
            t_val = acc.get();
        }
    }

    // 4. combine rows crossing thread boundaries (owner thread sums in thread order)
    __syncthreads();
    int64_t* s_hrow = reinterpret_cast<int64_t*>(s_raw);
    int64_t* s_trow = s_hrow + B;
    T* s_hval = reinterpret_cast<T*>(s_trow + B);
    T* s_tval = s_hval + B;
    s_hrow[tid] = h_row;
    s_trow[tid] = t_row;
    s_hval[tid] = h_val;
    s_tval[tid] = t_val;
    __syncthreads();
    if (t_row >= 0) {
        Sum<T> sum;
        sum.add(t_val);
        int u = tid + 1;
        while (u < B && s_hrow[u] == t_row) {
            sum.add(s_hval[u]);
            ++u;
        }
        const int64_t row_end = off[t_row - r_lo + 1];
        if (row_end <= ce) {
            if (t_row < a.row_limit) a.y[t_row] = epi(sum.get(), t_row);
        } else {
            a.tail[c] = sum.get();
            split_arrive_scalar(t_row, c, (row_end - 1) / S, a.cnt, a.head, a.tail, a.y, epi, a.row_limit);
        }
    }
    if (tid == 0 && s_hrow[0] >= 0) {
        const int64_t H = s_hrow[0];
        Sum<T> sum;
        sum.add(s_hval[0]);
        int u = 1;
        while (u < B && s_hrow[u] == H) {
            sum.add(s_hval[u]);
            ++u;
        }
        a.head[c] = sum.get();
        const int64_t jh = H - r_lo;
        split_arrive_scalar(H, off[jh] / S, (off[jh + 1] - 1) / S, a.cnt, a.head, a.tail, a.y, epi, a.row_limit);
    }
}

// ------------------------------------------------------------------ small kernels
template <typename T, bool AXPY>
__global__ void fill_rows_kernel(T* y, int64_t rows, int64_t row_limit, Epi<T, AXPY> epi) {
    for (int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; r < rows && r < row_limit;
         r += (int64_t)gridDim.x * blockDim.x)
        y[r] = epi(T(0), r);
}

__global__ void axpy_kernel(const double* __restrict__ x, const double* __restrict__ w, double* __restrict__ z,
                            double alpha, double beta, int64_t n) {
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
    if (s.split != TG_SPLIT_MERGE || nnz <= 0) return 0;
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
    if (s.split == TG_SPLIT_MERGE || s.split == TG_SPLIT_STREAM) {
        // stream needs 16-byte aligned operands; the merge split handles any alignment
        const int B = merge_block(s);
        const int64_t S = merge_chunk_nnz(B);
        const int64_t nchunks = ceil_div(A.nnz, S);
        const size_t need = split_ws_bytes(nchunks, 1, sizeof(T));
        if (ws == nullptr || ws_bytes < need)
            return set_error(TG_ENOMEM, "spmv merge split needs %zu workspace bytes, got %zu", need, ws_bytes);
        SplitWs w = split_ws_carve(ws, nchunks, 1, sizeof(T));
        int rc = launch_partition(A.indptr, A.rows, A.nnz, S, w, st);
        if (rc != TG_OK) return rc;
        a.own_first = w.own_first;
        a.cnt = w.cnt;
        a.head = static_cast<T*>(w.head);
        a.tail = static_cast<T*>(w.tail);
        a.err = w.err;
        a.use_bulk = aligned16(A.indices) && aligned16(A.data);
        if (nchunks > 0x7fffffff) return set_error(TG_EINVAL, "too many chunks (%lld)", (long long)nchunks);
        if (B == 128)
            spmv_merge_kernel<T, AXPY, 128><<<(unsigned)nchunks, 128, 0, st>>>(a, epi);
        else
            spmv_merge_kernel<T, AXPY, 256><<<(unsigned)nchunks, 256, 0, st>>>(a, epi);
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

int axpy_run(const double* x, const double* w, double* z, double alpha, double beta, int64_t n, int block,
             cudaStream_t st) {
    if (n == 0) return TG_OK;
    int64_t blocks = std::min<int64_t>(ceil_div(n, block), 148 * 16);
    axpy_kernel<<<(unsigned)blocks, block, 0, st>>>(x, w, z, alpha, beta, n);
    return check_launch("axpy_kernel");
}

}  // namespace tg
