// Streaming CSR SpMV for sm_100a: persistent, warp-specialised, TMA-fed row blocks.
//
// Same arithmetic as the reference's scalar_reduce kernels (tilegen/codegen.py:592-643,
// math cpp/src/ref.cpp:6-15 / :62-73), organised so that the CSR stream never touches the
// SM's load/store path:
//
//  * The rows are cut into ROW BLOCKS: block c holds the rows whose first nonzero lies in
//    positions [c*S, (c+1)*S) (the partition table own_first, tg_split.cuh), so a block
//    has about S nonzeros and no row is shared by two blocks.  Every CTA owns a
//    contiguous range of blocks (grid = SMs x CTAs per SM, persistent).
//  * Warp 8 is the producer: for each block it issues 1-D TMA bulk copies
//    (cp.async.bulk, no multicast) of the block's column indices, values and row
//    offsets into an NS-stage shared-memory ring, completion counted on the stage's
//    `full` mbarrier.  Block bounds come from own_first and indptr, loaded 32 blocks at a
//    time and prefetched half a batch ahead.
//  * Warps 0-7 consume: groups of TPR lanes take the block's rows round-robin, read the
//    row's indices and values from shared memory (consecutive lanes, consecutive
//    words), gather x from L2 and reduce with the group's own shuffle mask; the row's
//    result is written at once.  Each consumer warp releases the stage by arriving on
//    its `empty` mbarrier (8 arrivals), so warps never wait for one another.
//  * A block larger than a stage (a row longer than about S) is read from global memory
//    by the same consumer code; it stays correct, only slower (power-law matrices
//    belong to the merge split).
//
// Epilogues: plain y = A x, fused z = alpha A x + beta w, and the power-iteration step
// y = (A x) / sqrt(sum of the input slots) with sum(y^2) written to the output slot,
// reduced in a fixed order (per thread, fixed shuffle tree, CTAs in order by the last
// CTA to finish): results are deterministic.
#include <algorithm>
#include <mutex>
#include <set>

#include "tg_split.cuh"

namespace tg {

constexpr int kStreamConsumers = 256;  // 8 consumer warps
constexpr int kStreamThreads = kStreamConsumers + 32;
constexpr int kStreamMaxGrid = 148 * 4;

enum StreamMode { kPlain = 0, kAxpy = 1, kPower = 2 };

template <typename T>
struct StreamArgs {
    const int64_t* indptr;
    const int64_t* indices;
    const T* data;
    const T* x;
    T* y;
    int64_t rows;
    int64_t nnz;
    int64_t nchunks;
    int64_t row_limit;
    const int64_t* own_first;
    double* norm_part;
    unsigned* ticket;
    uint32_t* err;
    const T* w;
    T alpha, beta;
    int nparts;      // power: slots of x at r*stride + stride-1
    int64_t stride;  // power: output slot at y[stride-1]
};

template <typename T, int S, int NS>
struct StreamLayout {
    static constexpr int BUF = S + 128;         // nonzeros per stage (a block plus its overhang)
    static constexpr int ROWCAP = S / 4 + 66;   // row offsets per stage (even)
    static constexpr size_t kIdx = 0;
    static constexpr size_t kVal = kIdx + sizeof(int64_t) * BUF * NS;
    static constexpr size_t kOff = kVal + ((sizeof(T) * BUF * NS + 127) / 128) * 128;
    static constexpr size_t kMeta = kOff + sizeof(int64_t) * ROWCAP * NS;
    static constexpr int kMetaWords = 6;  // a (nnz base), nnz mode, ar (row base), row mode, of0, of1
    static constexpr size_t kBar = kMeta + sizeof(int64_t) * kMetaWords * NS;
    static constexpr size_t kBytes = kBar + sizeof(uint64_t) * 2 * NS;
};

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

template <typename T, int MODE>
__device__ __forceinline__ T stream_epi(const StreamArgs<T>& a, T acc, int64_t r, T scale) {
    if constexpr (MODE == kAxpy) {
        return a.alpha * acc + a.beta * a.w[r];
    } else if constexpr (MODE == kPower) {
        return scale * acc;
    } else {
        return acc;
    }
}

template <typename T, int MODE, int TPR, int S, int NS>
__global__ void __launch_bounds__(kStreamThreads, 2) spmv_stream_kernel(StreamArgs<T> a) {
    using L = StreamLayout<T, S, NS>;
    extern __shared__ __align__(128) unsigned char smem[];
    int64_t* s_idx = reinterpret_cast<int64_t*>(smem + L::kIdx);
    T* s_val = reinterpret_cast<T*>(smem + L::kVal);
    int64_t* s_off = reinterpret_cast<int64_t*>(smem + L::kOff);
    int64_t* s_meta = reinterpret_cast<int64_t*>(smem + L::kMeta);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kBar);
    uint64_t* empty = full + NS;
    __shared__ double s_red[8];
    __shared__ T s_scale;

    const int tid = threadIdx.x;
    const int64_t G = gridDim.x;
    const int64_t b = blockIdx.x;
    const int64_t k0 = b * a.nchunks / G;
    const int64_t k1 = (b + 1) * a.nchunks / G;

    if (tid == 0) {
        for (int st = 0; st < NS; ++st) {
            mbar_init(&full[st], 1);
            mbar_init(&empty[st], kStreamConsumers / 32);
        }
        fence_mbar_init();
        T sc = T(1);
        if constexpr (MODE == kPower) {
            double t = 0.0;
            for (int r = 0; r < a.nparts; ++r) t += (double)a.x[(int64_t)r * a.stride + a.stride - 1];
            sc = t > 0.0 ? T(1.0 / sqrt(t)) : T(0);
        }
        s_scale = sc;
    }
    __syncthreads();

    if (tid >= kStreamConsumers) {
        // ------------------------------------------------------------ producer warp
        const int lane = tid - kStreamConsumers;
        const uint64_t ps = policy_evict_first();
        constexpr int64_t gran = sizeof(T) == 4 ? 4 : 2;  // 16-byte granule of both arrays
        // batch of 32 blocks: lane l holds own_first[kb+l] and indptr[own_first[kb+l]]
        auto load_batch = [&](int64_t kb, int64_t& of, int64_t& pv, int64_t& of32, int64_t& pv32) {
            const int64_t kk = min(kb + lane, a.nchunks);
            of = a.own_first[kk];
            pv = a.indptr[of];
            const int64_t k32 = min(kb + 32, a.nchunks);
            of32 = a.own_first[k32];
            pv32 = a.indptr[of32];
        };
        int64_t kb = k0, of = 0, pv = 0, of32 = 0, pv32 = 0;
        int64_t nof = 0, npv = 0, nof32 = 0, npv32 = 0;
        bool have_next = false;
        if (k0 < k1) load_batch(kb, of, pv, of32, pv32);
        for (int64_t k = k0; k < k1; ++k) {
            const int64_t i = k - k0;
            const int stage = (int)(i % NS);
            int j = (int)(k - kb);
            if (j == 32) {  // next batch: prefetched at j == 16, else load it now
                kb += 32;
                j = 0;
                if (have_next) {
                    of = nof, pv = npv, of32 = nof32, pv32 = npv32;
                } else {
                    load_batch(kb, of, pv, of32, pv32);
                }
                have_next = false;
            }
            if (j == 16 && kb + 32 < k1) {
                load_batch(kb + 32, nof, npv, nof32, npv32);
                have_next = true;
            }
            const int64_t of0 = __shfl_sync(kFull, of, j);
            const int64_t p0 = __shfl_sync(kFull, pv, j);
            const int64_t of1 = j + 1 < 32 ? __shfl_sync(kFull, of, j + 1) : of32;
            const int64_t p1 = j + 1 < 32 ? __shfl_sync(kFull, pv, j + 1) : pv32;
            if (lane == 0) {
                if (i >= NS && !mbar_wait(&empty[stage], (uint32_t)(((i / NS) - 1) & 1))) atomicOr(a.err, 2u);
                int64_t* meta = s_meta + (int64_t)stage * L::kMetaWords;
                uint32_t bytes = 0;
                // nonzeros [p0, p1): from the 16-byte granule at or below p0
                const int64_t ab = p0 & ~(gran - 1);
                const int64_t n = p1 - ab;
                int64_t nmode = 0;  // 0: staged, 1: read from global memory
                int64_t nb = 0;
                if (n > L::BUF) {
                    nmode = 1;
                } else {
                    nb = n & ~(gran - 1);
                    for (int64_t q = nb; q < n; ++q) {  // ragged tail: plain loads
                        s_idx[(int64_t)stage * L::BUF + q] = a.indices[ab + q];
                        s_val[(int64_t)stage * L::BUF + q] = a.data[ab + q];
                    }
                    bytes += (uint32_t)(nb * 8 + nb * sizeof(T));
                }
                // row offsets indptr[of0 .. of1]
                const int64_t ar = of0 & ~int64_t(1);
                const int64_t nr = of1 + 1 - ar;
                int64_t rmode = 0;
                int64_t nrb = 0;
                if (nr > L::ROWCAP) {
                    rmode = 1;
                } else {
                    nrb = nr & ~int64_t(1);
                    if (nrb < nr) s_off[(int64_t)stage * L::ROWCAP + nr - 1] = a.indptr[ar + nr - 1];
                    bytes += (uint32_t)(nrb * 8);
                }
                meta[0] = ab;
                meta[1] = nmode;
                meta[2] = ar;
                meta[3] = rmode;
                meta[4] = of0;
                meta[5] = of1;
                mbar_arrive_expect_tx(&full[stage], bytes);
                if (nb > 0) {
                    bulk_g2s(s_idx + (int64_t)stage * L::BUF, a.indices + ab, (uint32_t)(nb * 8), &full[stage], ps);
                    bulk_g2s(s_val + (int64_t)stage * L::BUF, a.data + ab, (uint32_t)(nb * sizeof(T)), &full[stage],
                             ps);
                }
                if (nrb > 0)
                    bulk_g2s(s_off + (int64_t)stage * L::ROWCAP, a.indptr + ar, (uint32_t)(nrb * 8), &full[stage], ps);
            }
            __syncwarp();
        }
    } else {
        // ------------------------------------------------------------ consumer warps
        const uint64_t pg = policy_evict_last();
        const T scale = s_scale;
        const int lane = tid % TPR;
        const int group = tid / TPR;
        constexpr int kGroups = kStreamConsumers / TPR;
        unsigned gmask = kFull;
        if constexpr (TPR < 32) gmask = ((1u << TPR) - 1u) << ((tid % 32) / TPR * TPR);
        double sq = 0.0;
        for (int64_t k = k0; k < k1; ++k) {
            const int64_t i = k - k0;
            const int stage = (int)(i % NS);
            if (!mbar_wait(&full[stage], (uint32_t)((i / NS) & 1))) atomicOr(a.err, 1u);
            const int64_t* meta = s_meta + (int64_t)stage * L::kMetaWords;
            const int64_t ab = meta[0], ar = meta[2], of0 = meta[4], of1 = meta[5];
            const bool ng = meta[1] != 0, rg = meta[3] != 0;
            const int64_t* sidx = ng ? a.indices + ab : s_idx + (int64_t)stage * L::BUF;
            const T* sval = ng ? a.data + ab : s_val + (int64_t)stage * L::BUF;
            const int64_t* off = rg ? a.indptr + ar : s_off + (int64_t)stage * L::ROWCAP;
            for (int64_t r = of0 + group; r < of1; r += kGroups) {
                const int64_t q0 = off[r - ar] - ab;
                const int64_t q1 = off[r + 1 - ar] - ab;
                Sum<T> acc;
                int64_t q = q0 + lane;
                for (; q + 3 * TPR < q1; q += 4 * TPR) {  // four gathers in flight per lane
                    const int64_t c0 = sidx[q], c1 = sidx[q + TPR], c2 = sidx[q + 2 * TPR], c3 = sidx[q + 3 * TPR];
                    const T x0 = ld_gather(a.x + c0, pg), x1 = ld_gather(a.x + c1, pg);
                    const T x2 = ld_gather(a.x + c2, pg), x3 = ld_gather(a.x + c3, pg);
                    acc.mad(sval[q], x0);
                    acc.mad(sval[q + TPR], x1);
                    acc.mad(sval[q + 2 * TPR], x2);
                    acc.mad(sval[q + 3 * TPR], x3);
                }
                for (; q < q1; q += TPR) acc.mad(sval[q], ld_gather(a.x + sidx[q], pg));
                T v = acc.get();
                if constexpr (TPR > 1) v = group_sum<TPR>(v, gmask);
                if (lane == 0 && r < a.row_limit) {
                    const T out = stream_epi<T, MODE>(a, v, r, scale);
                    a.y[r] = out;
                    if constexpr (MODE == kPower) sq = fma((double)out, (double)out, sq);
                }
            }
            __syncwarp();
            if ((tid & 31) == 0) mbar_arrive(&empty[stage]);
        }
        double v = sq;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
        if ((tid & 31) == 0) s_red[tid >> 5] = v;
    }
    __syncthreads();
    // ---------------------------------------------------------------- norm (power)
    __shared__ bool s_last;
    if (tid == 0) {
        double part = 0.0;
        for (int w = 0; w < 8; ++w) part += s_red[w];
        a.norm_part[b] = part;
        __threadfence();
        s_last = (atomicAdd(a.ticket, 1u) == (unsigned)(G - 1));
    }
    __syncthreads();
    if (s_last && tid < 32) {
        __threadfence();
        double t = 0.0;
        for (int64_t c = tid; c < G; c += 32) t += __ldcg(&a.norm_part[c]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(kFull, t, o);
        if (tid == 0) {
            if constexpr (MODE == kPower) a.y[a.stride - 1] = (T)t;
            *a.ticket = 0u;
        }
    }
}

// ------------------------------------------------------------------ host side
namespace {

std::mutex g_attr_mu;
std::set<std::pair<const void*, int>> g_attr_done;

template <typename T, int MODE, int TPR, int S, int NS>
int launch_stream_inst(const StreamArgs<T>& a, int max_ctas_per_sm, cudaStream_t st) {
    using L = StreamLayout<T, S, NS>;
    auto fn = spmv_stream_kernel<T, MODE, TPR, S, NS>;
    int dev = 0;
    cudaGetDevice(&dev);
    int sms = 148;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    {
        std::lock_guard<std::mutex> lk(g_attr_mu);
        auto key = std::make_pair((const void*)fn, dev);
        if (!g_attr_done.count(key)) {
            int rc = check_cuda(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)L::kBytes),
                                "cudaFuncSetAttribute(stream smem)");
            if (rc != TG_OK) return rc;
            g_attr_done.insert(key);
        }
    }
    // persistent grid: every CTA resident at once
    int per_sm = 1;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, kStreamThreads, L::kBytes);
    per_sm = std::max(1, std::min(per_sm, max_ctas_per_sm));
    int64_t g = std::min<int64_t>(std::min<int64_t>(a.nchunks, (int64_t)sms * per_sm), kStreamMaxGrid);
    fn<<<(unsigned)g, kStreamThreads, L::kBytes, st>>>(a);
    return check_launch("spmv_stream_kernel");
}

template <typename T, int MODE, int S, int NS>
int stream_tpr(int tpr, const StreamArgs<T>& a, int per_sm, cudaStream_t st) {
    switch (tpr) {
        case 8: return launch_stream_inst<T, MODE, 8, S, NS>(a, per_sm, st);
        case 16: return launch_stream_inst<T, MODE, 16, S, NS>(a, per_sm, st);
        case 32: return launch_stream_inst<T, MODE, 32, S, NS>(a, per_sm, st);
        default: return launch_stream_inst<T, MODE, 4, S, NS>(a, per_sm, st);
    }
}

}  // namespace

// Shapes of the stream kernel -- block size S (nonzeros of the partition chunk) and ring
// depth NS -- selected by the schedule's unroll knob; all fit two CTAs per SM in fp64
// except unroll 8 (one CTA, three stages of 2048).
struct StreamShape {
    int S, NS;
};
inline StreamShape stream_shape(const tg_sched& s) {
    if (s.unroll >= 8) return {2048, 3};
    if (s.unroll >= 4) return {512, 8};
    if (s.unroll >= 2) return {2048, 2};
    return {1024, 4};
}

int64_t stream_chunk_nnz(const tg_sched& s) { return stream_shape(s).S; }

size_t stream_ws_bytes(int64_t nnz, const tg_sched& s, size_t elem) {
    (void)elem;
    const int64_t S = stream_chunk_nnz(s);
    const int64_t nchunks = nnz > 0 ? ceil_div(nnz, S) : 0;
    return align256(sizeof(int64_t) * (nchunks + 1)) + align256(sizeof(double) * kStreamMaxGrid) + 256;
}

struct StreamWs {
    int64_t* own_first;
    double* norm_part;
    unsigned* ticket;
    uint32_t* err;
};

static StreamWs stream_ws_carve(void* base, int64_t nchunks) {
    char* p = static_cast<char*>(base);
    StreamWs w;
    w.own_first = reinterpret_cast<int64_t*>(p);
    p += align256(sizeof(int64_t) * (nchunks + 1));
    w.norm_part = reinterpret_cast<double*>(p);
    p += align256(sizeof(double) * kStreamMaxGrid);
    w.ticket = reinterpret_cast<unsigned*>(p);
    w.err = reinterpret_cast<uint32_t*>(p + sizeof(unsigned));
    return w;
}

// Analysis pass of the stream kernel: the partition table (row blocks of about S
// nonzeros), and the ticket / error words cleared (partition_kernel zeroes *err; the
// ticket is left at zero by every completed launch and zeroed here for a new plan).
int stream_plan(const tg_csr& A, const tg_sched& s, void* ws, size_t ws_bytes, cudaStream_t st) {
    const int64_t S = stream_chunk_nnz(s);
    const int64_t nchunks = ceil_div(A.nnz, S);
    const size_t need = stream_ws_bytes(A.nnz, s, 8);
    if (ws == nullptr || ws_bytes < need)
        return set_error(TG_ENOMEM, "stream split needs %zu workspace bytes, got %zu", need, ws_bytes);
    StreamWs w = stream_ws_carve(ws, nchunks);
    SplitWs sw{};
    sw.own_first = w.own_first;
    sw.err = w.err;
    int rc = check_cuda(cudaMemsetAsync(w.ticket, 0, sizeof(unsigned), st), "cudaMemsetAsync(ticket)");
    if (rc != TG_OK) return rc;
    return launch_partition(A.indptr, A.rows, A.nnz, S, sw, st);
}

template <typename T, int MODE>
int stream_run(const tg_csr& A, const T* x, T* y, const T* w, T alpha, T beta, int nparts, int64_t stride,
               const tg_sched& s, void* ws, size_t ws_bytes, cudaStream_t st) {
    if (A.rows == 0) return TG_OK;
    if (A.nnz == 0) return set_error(TG_EINVAL, "stream split needs nnz > 0");
    if ((reinterpret_cast<uintptr_t>(A.indices) | reinterpret_cast<uintptr_t>(A.data) |
         reinterpret_cast<uintptr_t>(A.indptr)) & 15u)
        return set_error(TG_EUNSUPPORTED, "stream split needs 16-byte aligned indptr/indices/data");
    if (!(s.flags & TG_FLAG_REUSE_PLAN)) {
        int rc = stream_plan(A, s, ws, ws_bytes, st);
        if (rc != TG_OK) return rc;
    } else if (ws == nullptr || ws_bytes < stream_ws_bytes(A.nnz, s, sizeof(T))) {
        return set_error(TG_ENOMEM, "stream split: workspace too small for the reused plan");
    }
    const StreamShape sh = stream_shape(s);
    const int64_t nchunks = ceil_div(A.nnz, (int64_t)sh.S);
    StreamWs wsp = stream_ws_carve(ws, nchunks);
    StreamArgs<T> a{};
    a.indptr = A.indptr;
    a.indices = A.indices;
    a.data = static_cast<const T*>(A.data);
    a.x = x;
    a.y = y;
    a.rows = A.rows;
    a.nnz = A.nnz;
    a.nchunks = nchunks;
    a.row_limit = (s.flags & TG_FLAG_INJECT_BUG) ? A.rows - 1 : A.rows;
    a.own_first = wsp.own_first;
    a.norm_part = wsp.norm_part;
    a.ticket = wsp.ticket;
    a.err = wsp.err;
    a.w = w;
    a.alpha = alpha;
    a.beta = beta;
    a.nparts = nparts;
    a.stride = stride;
    // block_size knob: 128 -> one CTA per SM, otherwise as many as fit (at most 2)
    const int per_sm = s.block_size <= 128 ? 1 : 2;
    const int tpr = s.threads_per_row;
    if (sh.S == 512) return stream_tpr<T, MODE, 512, 8>(tpr, a, per_sm, st);
    if (sh.S == 1024) return stream_tpr<T, MODE, 1024, 4>(tpr, a, per_sm, st);
    if (sh.NS == 3) return stream_tpr<T, MODE, 2048, 3>(tpr, a, per_sm, st);
    return stream_tpr<T, MODE, 2048, 2>(tpr, a, per_sm, st);
}

template int stream_run<double, kPlain>(const tg_csr&, const double*, double*, const double*, double, double, int,
                                        int64_t, const tg_sched&, void*, size_t, cudaStream_t);
template int stream_run<double, kAxpy>(const tg_csr&, const double*, double*, const double*, double, double, int,
                                       int64_t, const tg_sched&, void*, size_t, cudaStream_t);
template int stream_run<double, kPower>(const tg_csr&, const double*, double*, const double*, double, double, int,
                                        int64_t, const tg_sched&, void*, size_t, cudaStream_t);
template int stream_run<float, kPlain>(const tg_csr&, const float*, float*, const float*, float, float, int,
                                       int64_t, const tg_sched&, void*, size_t, cudaStream_t);
template int stream_run<float, kAxpy>(const tg_csr&, const float*, float*, const float*, float, float, int,
                                       int64_t, const tg_sched&, void*, size_t, cudaStream_t);

}  // namespace tg
