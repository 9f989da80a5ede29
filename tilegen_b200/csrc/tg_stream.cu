// Streaming CSR SpMV for sm_100a: persistent, warp-specialised, TMA-fed.
//
// Same arithmetic as the reference's scalar_reduce kernels (tilegen/codegen.py:592-643,
// math cpp/src/ref.cpp:6-15 / :62-73), organised for HBM streaming:
//
//  * The nonzeros are cut into chunks of S = 256*I positions and every CTA owns a
//    contiguous range of chunks (grid = min(chunks, SMs * CTAs per SM)).
//  * Warp 8 is the producer: one lane issues, per chunk, three 1-D TMA bulk copies
//    (cp.async.bulk, no multicast) -- the chunk's column indices, its values, and the
//    slice of indptr covering the rows that touch the chunk -- into an NS-stage ring of
//    shared-memory buffers, completion counted on the stage's `full` mbarrier.  The
//    row bounds of each chunk come from the partition table own_first (tg_split.cuh),
//    prefetched 32 chunks at a time by the producer warp.
//  * Warps 0-7 consume: each thread multiplies I consecutive nonzeros of the chunk
//    (all x gathers in flight together), then walks them against the staged row
//    offsets.  Rows crossing thread boundaries are summed by their owner thread; a row
//    crossing a chunk boundary is carried to the next chunk of the same CTA in shared
//    memory, so only the first and the last row of a CTA's range can be split across
//    CTAs.  Those are published per CTA and resolved, in CTA order, by the last CTA to
//    finish (atomic ticket), which is also where the power-iteration norm is reduced.
//    Every sum is taken in a fixed order: results are deterministic.
//
// Epilogues: plain y = A x, fused z = alpha A x + beta w, and the power-iteration step
// y = (A x) / sqrt(sum of the input slots) with sum(y^2) written to the output slot.
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
    // per-CTA split rows and norm partials (workspace)
    int64_t* head_row;
    int64_t* tail_row;
    T* head_val;
    T* tail_val;
    double* norm_part;
    unsigned* ticket;
    uint32_t* err;
    // epilogues
    const T* w;
    T alpha, beta;
    int nparts;       // power: slots of x at r*stride + stride-1
    int64_t stride;   // power: output slot at y[stride-1]
};

template <typename T, int I, int NS>
struct StreamLayout {
    static constexpr int S = kStreamConsumers * I;
    // row offsets staged per chunk (even); chunks touching more rows (mean row length
    // below ~4) read them from global memory instead
    static constexpr int OWCAP = S / 4 + 66;
    static constexpr size_t kIdx = 0;
    static constexpr size_t kVal = kIdx + sizeof(int64_t) * S * NS;
    static constexpr size_t kOff = kVal + ((sizeof(T) * S * NS + 127) / 128) * 128;
    static constexpr size_t kMeta = kOff + sizeof(int64_t) * OWCAP * NS;
    // meta: per stage off_base, off_n (int64), then full/empty barriers
    static constexpr size_t kBar = kMeta + sizeof(int64_t) * 2 * NS;
    static constexpr size_t kComb = ((kBar + sizeof(uint64_t) * 2 * NS + 127) / 128) * 128;
    // combine: hrow, trow (int64), hval, tval (T), red (double, 8 warps), carry
    static constexpr size_t kCarry = kComb + (2 * sizeof(int64_t) + 2 * sizeof(T)) * kStreamConsumers;
    static constexpr size_t kBytes = kCarry + 128;
};

__device__ __forceinline__ void consumer_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kStreamConsumers) : "memory"); }

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

template <typename T, int MODE, int I, int NS>
__global__ void __launch_bounds__(kStreamThreads, 1) spmv_stream_kernel(StreamArgs<T> a) {
    using L = StreamLayout<T, I, NS>;
    constexpr int S = L::S;
    extern __shared__ __align__(128) unsigned char smem[];
    int64_t* s_idx = reinterpret_cast<int64_t*>(smem + L::kIdx);
    T* s_val = reinterpret_cast<T*>(smem + L::kVal);
    int64_t* s_off = reinterpret_cast<int64_t*>(smem + L::kOff);
    int64_t* s_meta = reinterpret_cast<int64_t*>(smem + L::kMeta);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kBar);
    uint64_t* empty = full + NS;
    int64_t* s_hrow = reinterpret_cast<int64_t*>(smem + L::kComb);
    int64_t* s_trow = s_hrow + kStreamConsumers;
    T* s_hval = reinterpret_cast<T*>(s_trow + kStreamConsumers);
    T* s_tval = s_hval + kStreamConsumers;
    // carry state (thread 0 of the consumers owns it); next-tail slot written by owners
    int64_t* c_row = reinterpret_cast<int64_t*>(smem + L::kCarry);
    int64_t* c_next_row = c_row + 1;
    int* c_ctahead = reinterpret_cast<int*>(c_row + 2);
    T* c_val = reinterpret_cast<T*>(c_row + 4);
    T* c_next_val = c_val + 1;
    __shared__ double s_red[8];
    __shared__ T s_scale;
    __shared__ int s_fail;

    const int tid = threadIdx.x;
    const int64_t G = gridDim.x;
    const int64_t b = blockIdx.x;
    const int64_t k0 = b * a.nchunks / G;
    const int64_t k1 = (b + 1) * a.nchunks / G;
    const int64_t nk = k1 - k0;

    if (tid == 0) {
        for (int s = 0; s < NS; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        fence_mbar_init();
        *c_row = -1;
        *c_next_row = -1;
        *c_ctahead = 0;
        *c_val = T(0);
        s_fail = 0;
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
        int64_t ofbuf = 0;  // own_first[kb + lane] for the current batch of 32 chunks
        int64_t kb = -1;
        for (int64_t k = k0; k < k1; ++k) {
            const int64_t i = k - k0;
            const int stage = (int)(i % NS);
            if (k >= kb + 32 || kb < 0) {  // the table entries of chunks k .. k+32
                kb = k;
                ofbuf = (kb + lane <= a.nchunks) ? a.own_first[kb + lane] : a.rows;
            }
            int64_t of0 = __shfl_sync(kFull, ofbuf, (int)(k - kb));
            int64_t of1 = (k + 1 - kb < 32) ? __shfl_sync(kFull, ofbuf, (int)(k + 1 - kb)) : a.own_first[k + 1];
            if (lane == 0) {
                if (i >= NS && !mbar_wait(&empty[stage], (uint32_t)(((i / NS) - 1) & 1))) {
                    atomicOr(a.err, 2u);
                    s_fail = 1;
                }
                const int64_t cs = k * S;
                const int64_t ce = min(cs + (int64_t)S, a.nnz);
                const int64_t n = ce - cs;
                constexpr int64_t gran = sizeof(T) == 4 ? 4 : 2;
                const int64_t nbulk = (n / gran) * gran;
                // row offsets indptr[rlo .. of1] covering every row that touches the chunk
                const int64_t rlo = of0 > 0 ? of0 - 1 : 0;
                const int64_t a0 = rlo & ~int64_t(1);
                int64_t noff = of1 + 1 - a0;  // entries a0 .. of1
                int64_t* off_dst = s_off + (int64_t)stage * L::OWCAP;
                uint32_t bytes = (uint32_t)(nbulk * 8 + nbulk * sizeof(T));
                int64_t off_n = -noff;  // negative: read the offsets from global memory
                int64_t nb_off = 0;
                if (noff <= L::OWCAP) {
                    nb_off = noff & ~int64_t(1);
                    off_n = noff;
                    bytes += (uint32_t)(nb_off * 8);
                }
                // scalar leftovers first (plain shared stores are released by the arrive)
                for (int64_t q = nbulk; q < n; ++q) {
                    s_idx[(int64_t)stage * S + q] = a.indices[cs + q];
                    s_val[(int64_t)stage * S + q] = a.data[cs + q];
                }
                if (off_n > 0 && nb_off < noff) off_dst[noff - 1] = a.indptr[a0 + noff - 1];
                s_meta[2 * stage] = a0;
                s_meta[2 * stage + 1] = off_n;
                mbar_arrive_expect_tx(&full[stage], bytes);
                if (nbulk > 0) {
                    bulk_g2s(s_idx + (int64_t)stage * S, a.indices + cs, (uint32_t)(nbulk * 8), &full[stage], ps);
                    bulk_g2s(s_val + (int64_t)stage * S, a.data + cs, (uint32_t)(nbulk * sizeof(T)), &full[stage], ps);
                }
                if (nb_off > 0) bulk_g2s(off_dst, a.indptr + a0, (uint32_t)(nb_off * 8), &full[stage], ps);
            }
            __syncwarp();
        }
    } else {
        // ------------------------------------------------------------ consumer warps
        const uint64_t pg = policy_evict_last();
        const T scale = s_scale;
        double sq = 0.0;  // power: sum of squares of the rows this thread wrote
        // x gathers run one chunk ahead of the walk: xn holds chunk k+1's values (loads in
        // flight) while chunk k is walked, so the L2 gather latency overlaps the walk.
        T xn[I];
        auto gather = [&](int64_t kc, int st) {
            const int64_t ccs = kc * S;
            const int64_t cce = min(ccs + (int64_t)S, a.nnz);
            const int64_t* gi = s_idx + (int64_t)st * S;
#pragma unroll
            for (int kk = 0; kk < I; ++kk) {
                const int64_t q = ccs + (int64_t)tid * I + kk;
                xn[kk] = T(0);
                if (q < cce) xn[kk] = ld_gather(a.x + gi[q - ccs], pg);
            }
        };
        if (nk > 0) {
            if (!mbar_wait(&full[0], 0u)) {
                atomicOr(a.err, 1u);
                s_fail = 1;
            }
            gather(k0, 0);
        }
        for (int64_t k = k0; k < k1; ++k) {
            const int64_t i = k - k0;
            const int stage = (int)(i % NS);
            T xc[I];
#pragma unroll
            for (int kk = 0; kk < I; ++kk) xc[kk] = xn[kk];
            // start chunk k+1's gathers now if its data has landed, else after this walk
            const int st1 = (int)((i + 1) % NS);
            const uint32_t ph1 = (uint32_t)(((i + 1) / NS) & 1);
            bool next_started = false;
            if (k + 1 < k1 && mbar_test(&full[st1], ph1)) {
                gather(k + 1, st1);
                next_started = true;
            }
            const int64_t cs = k * S;
            const int64_t ce = min(cs + (int64_t)S, a.nnz);
            const int64_t a0 = s_meta[2 * stage];
            const int64_t off_n = s_meta[2 * stage + 1];
            const int64_t* off = off_n > 0 ? s_off + (int64_t)stage * L::OWCAP : a.indptr + a0;
            const int64_t n_off = off_n > 0 ? off_n : -off_n;
            const T* sval = s_val + (int64_t)stage * S;

            const int64_t qa = cs + (int64_t)tid * I;
            const int64_t qb = min(qa + (int64_t)I, ce);
            int64_t h_row = -1, t_row = -1;
            T h_val = T(0), t_val = T(0);
            if (qa < qb) {
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
                for (int kk = 0; kk < I; ++kk) {
                    const int64_t q = qa + kk;
                    if (q < qb) {
                        while (nxt <= q) {
                            const int64_t r = a0 + j;
                            if (first && head) {
                                h_row = r;
                                h_val = acc.get();
                            } else if (r < a.row_limit) {
                                const T v = stream_epi<T, MODE>(a, acc.get(), r, scale);
                                a.y[r] = v;
                                if constexpr (MODE == kPower) sq = fma((double)v, (double)v, sq);
                            }
                            first = false;
                            acc = Sum<T>();
                            ++j;
                            nxt = off[j + 1];
                        }
                        acc.add(sval[q - cs] * xc[kk]);
                    }
                }
                const int64_t r = a0 + j;
                if (nxt == qb) {
                    if (first && head) {
                        h_row = r;
                        h_val = acc.get();
                    } else if (r < a.row_limit) {
                        const T v = stream_epi<T, MODE>(a, acc.get(), r, scale);
                        a.y[r] = v;
                        if constexpr (MODE == kPower) sq = fma((double)v, (double)v, sq);
                    }
                    if (qb == a.nnz)
                        for (int64_t rr = r + 1; rr < a.rows && rr < a.row_limit; ++rr) {
                            a.y[rr] = stream_epi<T, MODE>(a, T(0), rr, scale);
                        }
                } else if (first && head) {
                    h_row = r;
                    h_val = acc.get();
                } else {
                    t_row = r;
                    t_val = acc.get();
                }
            }
            if (k + 1 < k1 && !next_started) {
                if (!mbar_wait(&full[st1], ph1)) {
                    atomicOr(a.err, 1u);
                    s_fail = 1;
                }
                gather(k + 1, st1);
            }
            s_hrow[tid] = h_row;
            s_trow[tid] = t_row;
            s_hval[tid] = h_val;
            s_tval[tid] = t_val;
            consumer_sync();
            // rows crossing thread boundaries: the owner (the thread where the row started)
            if (t_row >= 0) {
                Sum<T> sum;
                sum.add(t_val);
                int u = tid + 1;
                while (u < kStreamConsumers && s_hrow[u] == t_row) {
                    sum.add(s_hval[u]);
                    ++u;
                }
                const int64_t row_end = off[t_row - a0 + 1];
                if (row_end <= ce) {
                    if (t_row < a.row_limit) {
                        const T v = stream_epi<T, MODE>(a, sum.get(), t_row, scale);
                        a.y[t_row] = v;
                        if constexpr (MODE == kPower) sq = fma((double)v, (double)v, sq);
                    }
                } else {  // continues into the next chunk: the new carry
                    *c_next_row = t_row;
                    *c_next_val = sum.get();
                }
            }
            // the chunk's head row (started before cs) meets the carry of the previous chunk
            if (tid == 0) {
                const int64_t H = s_hrow[0];
                if (H >= 0) {
                    Sum<T> sum;
                    sum.add(s_hval[0]);
                    int u = 1;
                    while (u < kStreamConsumers && s_hrow[u] == H) {
                        sum.add(s_hval[u]);
                        ++u;
                    }
                    T total = sum.get();
                    bool ctahead = true;  // started before this CTA's range unless carried
                    if (*c_row == H) {
                        Sum<T> t2;
                        t2.add(*c_val);
                        t2.add(total);
                        total = t2.get();
                        ctahead = *c_ctahead != 0;
                    }
                    const int64_t row_end = off[H - a0 + 1];
                    if (row_end <= ce) {
                        if (ctahead) {
                            a.head_row[b] = H;
                            a.head_val[b] = total;
                        } else if (H < a.row_limit) {
                            const T v = stream_epi<T, MODE>(a, total, H, scale);
                            a.y[H] = v;
                            if constexpr (MODE == kPower) sq = fma((double)v, (double)v, sq);
                        }
                        *c_row = -1;
                    } else {  // through: keeps going into the next chunk
                        *c_row = H;
                        *c_val = total;
                        *c_ctahead = ctahead ? 1 : 0;
                    }
                }
            }
            consumer_sync();
            if (tid == 0) {
                if (*c_next_row >= 0) {
                    *c_row = *c_next_row;
                    *c_val = *c_next_val;
                    *c_ctahead = 0;
                    *c_next_row = -1;
                }
                mbar_arrive(&empty[stage]);
            }
        }
        // the row still open at the end of the range crosses into the next CTA
        if (tid == 0 && nk > 0 && *c_row >= 0) {
            if (*c_ctahead) {
                a.head_row[b] = *c_row;
                a.head_val[b] = *c_val;
            } else {
                a.tail_row[b] = *c_row;
                a.tail_val[b] = *c_val;
            }
        }
        // per-CTA norm partial (fixed shuffle tree, warps in order)
        double v = sq;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
        if ((tid & 31) == 0) s_red[tid >> 5] = v;
    }
    __syncthreads();
    __shared__ bool s_last;
    if (tid == 0) {
        double part = 0.0;
        for (int w = 0; w < 8; ++w) part += s_red[w];
        a.norm_part[b] = part;
        __threadfence();
        s_last = (atomicAdd(a.ticket, 1u) == (unsigned)(G - 1));
    }
    __syncthreads();
    if (!s_last) return;
    // ---------------------------------------------------------------- last CTA
    __threadfence();
    double sq2 = 0.0;
    if (tid < kStreamConsumers) {
        const T scale = s_scale;
        for (int64_t c = tid; c < G; c += kStreamConsumers) {
            const int64_t R = __ldcg(&a.tail_row[c]);
            if (R < 0) continue;
            Sum<T> sum;
            sum.add(ld_cg(&a.tail_val[c]));
            for (int64_t c2 = c + 1; c2 < G && __ldcg(&a.head_row[c2]) == R; ++c2) sum.add(ld_cg(&a.head_val[c2]));
            if (R < a.row_limit) {
                const T v = stream_epi<T, MODE>(a, sum.get(), R, scale);
                a.y[R] = v;
                if constexpr (MODE == kPower) sq2 = fma((double)v, (double)v, sq2);
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sq2 += __shfl_xor_sync(kFull, sq2, o);
        if ((tid & 31) == 0) s_red[tid >> 5] = sq2;
    }
    __syncthreads();
    if (tid < 32) {
        double t = 0.0;
        for (int64_t c = tid; c < G; c += 32) t += __ldcg(&a.norm_part[c]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(kFull, t, o);
        if (tid == 0) {
            for (int w = 0; w < 8; ++w) t += s_red[w];
            if constexpr (MODE == kPower) a.y[a.stride - 1] = (T)t;
            *a.ticket = 0u;
        }
    }
    // reset the split-row slots for the next call on this workspace (after every read)
    __syncthreads();
    for (int64_t c = tid; c < G; c += blockDim.x) {
        a.head_row[c] = -1;
        a.tail_row[c] = -1;
    }
}

// ------------------------------------------------------------------ host side
namespace {

std::mutex g_attr_mu;
std::set<std::pair<const void*, int>> g_attr_done;

template <typename T, int MODE, int I, int NS>
int launch_stream_inst(const StreamArgs<T>& a, int max_ctas_per_sm, cudaStream_t st) {
    using L = StreamLayout<T, I, NS>;
    auto fn = spmv_stream_kernel<T, MODE, I, NS>;
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

}  // namespace

// Chunk shapes of the stream kernel: items per thread I (odd: conflict-free smem) and
// ring depth NS, selected by the schedule's unroll knob.
struct StreamShape {
    int I, NS;
};
inline StreamShape stream_shape(const tg_sched& s) {
    if (s.unroll >= 8) return {3, 6};
    if (s.unroll >= 4) return {5, 4};
    if (s.unroll >= 2) return {7, 3};
    return {5, 3};
}

int64_t stream_chunk_nnz(const tg_sched& s) { return (int64_t)kStreamConsumers * stream_shape(s).I; }

size_t stream_ws_bytes(int64_t nnz, const tg_sched& s, size_t elem) {
    const int64_t S = stream_chunk_nnz(s);
    const int64_t nchunks = nnz > 0 ? ceil_div(nnz, S) : 0;
    return align256(sizeof(int64_t) * (nchunks + 1)) + 4 * align256(8 * kStreamMaxGrid) +
           align256(sizeof(double) * kStreamMaxGrid) + align256(sizeof(unsigned) + sizeof(uint32_t)) +
           0 * elem;
}

struct StreamWs {
    int64_t* own_first;
    int64_t* head_row;
    int64_t* tail_row;
    void* head_val;
    void* tail_val;
    double* norm_part;
    unsigned* ticket;
    uint32_t* err;
};

static StreamWs stream_ws_carve(void* base, int64_t nchunks) {
    char* p = static_cast<char*>(base);
    StreamWs w;
    w.own_first = reinterpret_cast<int64_t*>(p);
    p += align256(sizeof(int64_t) * (nchunks + 1));
    w.head_row = reinterpret_cast<int64_t*>(p);
    p += align256(8 * kStreamMaxGrid);
    w.tail_row = reinterpret_cast<int64_t*>(p);
    p += align256(8 * kStreamMaxGrid);
    w.head_val = p;
    p += align256(8 * kStreamMaxGrid);
    w.tail_val = p;
    p += align256(8 * kStreamMaxGrid);
    w.norm_part = reinterpret_cast<double*>(p);
    p += align256(sizeof(double) * kStreamMaxGrid);
    w.ticket = reinterpret_cast<unsigned*>(p);
    w.err = reinterpret_cast<uint32_t*>(p + sizeof(unsigned));
    return w;
}

__global__ void stream_reset_kernel(int64_t* head_row, int64_t* tail_row, unsigned* ticket, uint32_t* err, int n) {
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        head_row[i] = -1;
        tail_row[i] = -1;
    }
    if (threadIdx.x == 0) {
        *ticket = 0u;
        *err = 0u;
    }
}

// Analysis pass of the stream kernel: the partition table of its chunk size, and the
// per-CTA slots reset.  Needed once per matrix / workspace (see TG_FLAG_REUSE_PLAN).
int stream_plan(const tg_csr& A, const tg_sched& s, void* ws, size_t ws_bytes, cudaStream_t st) {
    const int64_t S = stream_chunk_nnz(s);
    const int64_t nchunks = ceil_div(A.nnz, S);
    const size_t need = stream_ws_bytes(A.nnz, s, 8);
    if (ws == nullptr || ws_bytes < need)
        return set_error(TG_ENOMEM, "stream split needs %zu workspace bytes, got %zu", need, ws_bytes);
    StreamWs w = stream_ws_carve(ws, nchunks);
    SplitWs sw{};
    sw.own_first = w.own_first;  // no arrival counters: the stream kernel resolves splits itself
    int rc = launch_partition(A.indptr, A.rows, A.nnz, S, sw, st);
    if (rc != TG_OK) return rc;
    stream_reset_kernel<<<1, 256, 0, st>>>(w.head_row, w.tail_row, w.ticket, w.err, kStreamMaxGrid);
    return check_launch("stream_reset_kernel");
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
    const int64_t S = (int64_t)kStreamConsumers * sh.I;
    const int64_t nchunks = ceil_div(A.nnz, S);
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
    a.head_row = wsp.head_row;
    a.tail_row = wsp.tail_row;
    a.head_val = static_cast<T*>(wsp.head_val);
    a.tail_val = static_cast<T*>(wsp.tail_val);
    a.norm_part = wsp.norm_part;
    a.ticket = wsp.ticket;
    a.err = wsp.err;
    a.w = w;
    a.alpha = alpha;
    a.beta = beta;
    a.nparts = nparts;
    a.stride = stride;
    // block_size knob: 128 -> one CTA per SM, otherwise as many as fit (at most 2)
    const int max_per_sm = s.block_size <= 128 ? 1 : 2;
    if (sh.I == 3) return launch_stream_inst<T, MODE, 3, 6>(a, max_per_sm, st);
    if (sh.I == 5 && sh.NS == 4) return launch_stream_inst<T, MODE, 5, 4>(a, max_per_sm, st);
    if (sh.I == 7) return launch_stream_inst<T, MODE, 7, 3>(a, max_per_sm, st);
    return launch_stream_inst<T, MODE, 5, 3>(a, max_per_sm, st);
}

template int stream_run<double, kPlain>(const tg_csr&, const double*, double*, const double*, double, double, int,
                                        int64_t, const tg_sched&, void*, size_t, cudaStream_t);
template int stream_run<double, kAxpy>(const tg_csr&, const double*, double*, const double*, double, double, int,
                                       int64_t, const tg_sched&, void*, size_t, cudaStream_t);
template int stream_run<double, kPower>(const tg_csr&, const double*, double*, const double*, double, double, int,
                                        int64_t, const tg_sched&, void*, size_t, cudaStream_t);
template int stream_run<float, kPlain>(const tg_csr&, const float*, float*, const float*, float, float, int,
                                       int64_t, const tg_sched&, void*, size_t, cudaStream_t);

}  // namespace tg
