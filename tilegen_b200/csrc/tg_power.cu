// Power iteration x <- A x / ||A x|| on 1..8 GPUs (no counterpart in the reference: the
// iterated-SpMV mode is new; its SpMV is the rowwise kernel of tg_spmv.cu).
//
// Layout.  Rows are split into P contiguous shards; shard r of the iterate lives at
// x[r*stride, r*stride + rows_r) of a padded vector of P*stride doubles, and its last
// element x[r*stride + stride - 1] (the SLOT) holds sum(shard^2).  Column indices of a
// rank's rows are renumbered once to this padded layout, so the vector that an
// all-gather of the shards produces is directly the next x.
//
// One step (tg_power_step_f64) is one kernel: every CTA reads the P slots of the input
// iterate x~ and forms s = 1/sqrt(sum slots) (the normalisation of the previous step,
// applied lazily), computes y = s * (A_local x~) for its rows, writes y into the output
// shard, and reduces sum(y^2) into the output slot deterministically: per-thread sums in
// a fixed row order, a fixed block tree, one partial per CTA, and the last CTA to arrive
// (atomic ticket) adds the partials in CTA order.  No separate norm or scale pass.
#include <algorithm>
#include <mutex>
#include <vector>

#include "tg_rowdot.cuh"

namespace tg {

struct PowerArgs {
    const int64_t* indptr;
    const void* indices;  // renumbered to the padded layout: int64, or int32 (TG_FLAG_INDEX32)
    const double* data;
    const double* x;  // padded input iterate, nparts * stride
    int nparts;
    int64_t stride;
    double* y;  // output rows (the shard, or a chunk of its rows)
    int64_t rows;
    int64_t rows_per_tile;
    double* partials;  // [gridDim.x]
    unsigned* ticket;  // [1], zero between launches
    double* slot_out;  // where sum(y^2) goes: the shard's slot, or a chunk's partial
};

// Deterministic sum of per-thread values of one CTA (fixed shuffle tree, warps in order).
__device__ __forceinline__ double block_sum(double v, double* s_warp) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(kFull, v, off);
    const int w = threadIdx.x / 32;
    if ((threadIdx.x & 31) == 0) s_warp[w] = v;
    __syncthreads();
    double t = 0.0;
    if (threadIdx.x == 0) {
        const int nw = (blockDim.x + 31) / 32;
        for (int i = 0; i < nw; ++i) t += s_warp[i];
    }
    return t;  // valid in thread 0
}

// Called by every thread after its partial for this CTA is final (in thread 0): the last
// CTA to arrive sums all partials in CTA order into *out.
__device__ __forceinline__ void grid_sum_last(double part, double* partials, unsigned* ticket, double* out) {
    __shared__ bool s_last;
    if (threadIdx.x == 0) {
        partials[blockIdx.x] = part;
        __threadfence();
        const unsigned t = atomicAdd(ticket, 1u);
        s_last = (t == gridDim.x - 1);
    }
    __syncthreads();
    if (s_last && threadIdx.x < 32) {
        __threadfence();
        double v = 0.0;
        // lane l sums partials l, l+32, ... then a fixed shuffle tree
        for (unsigned i = threadIdx.x; i < gridDim.x; i += 32) v += __ldcg(&partials[i]);
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(kFull, v, off);
        if (threadIdx.x == 0) {
            *out = v;
            *ticket = 0u;
        }
    }
}

template <int TPR, int U, int V, typename I>
__global__ void __launch_bounds__(512) power_step_kernel(PowerArgs a) {
    const I* indices = static_cast<const I*>(a.indices);
    __shared__ double s_warp[32];
    __shared__ double s_scale;
    const uint64_t ps = policy_evict_first();
    const uint64_t pg = policy_evict_last();
    if (threadIdx.x == 0) {
        double t = 0.0;
        for (int r = 0; r < a.nparts; ++r) t += a.x[(int64_t)r * a.stride + a.stride - 1];
        s_scale = t > 0.0 ? 1.0 / sqrt(t) : 0.0;
    }
    __syncthreads();
    const double scale = s_scale;
    const int lane = threadIdx.x % TPR;
    const int group = threadIdx.x / TPR;
    const int groups = blockDim.x / TPR;
    unsigned mask = kFull;
    if constexpr (TPR < 32) mask = ((1u << TPR) - 1u) << ((threadIdx.x % 32) / TPR * TPR);
    double sq = 0.0;
    for (int64_t base = (int64_t)blockIdx.x * a.rows_per_tile; base < a.rows;
         base += (int64_t)gridDim.x * a.rows_per_tile) {
        const int64_t end = min(base + a.rows_per_tile, a.rows);
        for (int64_t i = base + group; i < end; i += groups) {
            double acc = row_dot<double, TPR, U, V, I, true>(indices, a.data, a.x, a.indptr[i], a.indptr[i + 1], lane, ps, pg);
            if constexpr (TPR > 1) acc = group_sum<TPR>(acc, mask);
            if (lane == 0) {
                const double v = scale * acc;
                a.y[i] = v;
                sq = fma(v, v, sq);
            }
        }
    }
    const double part = block_sum(sq, s_warp);
    grid_sum_last(part, a.partials, a.ticket, a.slot_out);
}

// ------------------------------------------------------------------ fused exchange
// The power step fused with the shard exchange over peer memory (1..8 GPUs, CUDA IPC
// mappings, plain P2P stores, no multicast).  Iteration `epoch` reads the local copy of
// the iterate x (all shards) and writes its own shard of the next iterate straight into
// every rank's next-iterate buffer y_peers[q] (own rank included), one tile of rows at a
// time, so the NVLink transfer overlaps the SpMV.  Protocol, per kernel:
//   1. wait (bounded, 2 s) until every rank's flag in the LOCAL flag array reached
//      epoch-1: all ranks finished the previous iteration, so the local x is complete
//      and nobody still reads the buffer this kernel writes;
//   2. rowwise SpMV of the tile, y = s * (A x) staged in shared memory, pushed to every
//      rank with coalesced 8-byte stores;
//   3. each CTA fences (system scope) and takes a ticket; the last CTA sums the norm
//      partials in CTA order, writes the slot to every rank, fences, and release-stores
//      `epoch` into flag_peers[q][rank] for every q.
// Failure (a peer that stops answering).  A wait that runs out sets bit 4 of *err.  The
// error word is sticky: a CTA that finds it set (at entry, or while it waits because
// another CTA gave up) skips its rows without waiting any longer, so a failed launch
// ends about 2 s after it started instead of 2 s per wave of CTAs.  Every CTA still
// takes its ticket, so the ticket returns to zero at the end of every launch, and the
// last CTA neither writes the slot nor publishes the epoch when *err is set: the peers
// see no flag and give up in turn.  The host reads *err (tg_power_error) and clears it
// (tg_power_clear_error) only after every rank agreed to restart from zeroed flags.
struct PowerP2PArgs {
    const int64_t* indptr;
    const void* indices;  // int64, or int32 (TG_FLAG_INDEX32)
    const double* data;
    const double* x;  // local padded iterate (nparts * stride)
    int nparts;
    int rank;
    int64_t stride;
    double* y_peers[8];          // next-iterate buffer of every rank (nparts * stride each)
    unsigned long long* flag_peers[8];  // flag array (nparts words) of every rank
    unsigned long long* flag_local;     // this rank's flag array
    unsigned long long epoch;
    int64_t rows;
    double* partials;
    unsigned* ticket;
    uint32_t* err;
};

__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void st_release_sys(unsigned long long* p, unsigned long long v) {
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_err(const uint32_t* p) { return *reinterpret_cast<const volatile uint32_t*>(p); }

// Bounded wait (2 s) until flag_local[q] >= need for every q < nparts.  Gives up at once
// when *err is already set; sets bit 4 of *err when the time runs out.  Returns whether
// the wait was met.
__device__ __forceinline__ bool wait_flags(const unsigned long long* flag_local, int nparts, unsigned long long need,
                                           uint32_t* err) {
    if (ld_err(err) != 0u) return false;
    const uint64_t t0 = globaltimer_ns();
    for (int q = 0; q < nparts; ++q) {
        while (ld_acquire_sys(&flag_local[q]) < need) {
            if (ld_err(err) != 0u) return false;  // another CTA (or an earlier launch) gave up
            if (globaltimer_ns() - t0 > 2000000000ull) {
                atomicOr(err, 16u);
                return false;
            }
        }
    }
    return true;
}

template <int TPR, int U, int V, typename I>
__global__ void __launch_bounds__(256) power_p2p_kernel(PowerP2PArgs a) {
    const I* indices = static_cast<const I*>(a.indices);
    constexpr int kGroups = 256 / TPR;  // rows per CTA tile: one per lane group
    constexpr int kWarpRows = 32 / TPR; // consecutive rows owned by one warp per tile
    __shared__ double s_warp[32];
    __shared__ double s_scale;
    __shared__ int s_ok;
    const uint64_t ps = policy_evict_first();
    const uint64_t pg = policy_evict_last();
    if (threadIdx.x == 0) {
        const int ok = wait_flags(a.flag_local, a.nparts, a.epoch - 1, a.err) ? 1 : 0;
        s_ok = ok;
        double t = 0.0;
        if (ok)
            for (int r = 0; r < a.nparts; ++r) t += a.x[(int64_t)r * a.stride + a.stride - 1];
        s_scale = t > 0.0 ? 1.0 / sqrt(t) : 0.0;
    }
    __syncthreads();
    __threadfence_system();
    const double scale = s_scale;
    const int lane = threadIdx.x % TPR;
    const int group = threadIdx.x / TPR;
    const int wl = threadIdx.x & 31;
    unsigned mask = kFull;
    if constexpr (TPR < 32) mask = ((1u << TPR) - 1u) << ((threadIdx.x % 32) / TPR * TPR);
    const int64_t own = (int64_t)a.rank * a.stride;
    double sq = 0.0;
    const int64_t rows = s_ok ? a.rows : 0;  // a CTA whose wait failed skips its rows
    for (int64_t base = (int64_t)blockIdx.x * kGroups; base < rows; base += (int64_t)gridDim.x * kGroups) {
        const int64_t i = base + group;
        double v = 0.0;
        if (i < rows) {
            double acc = row_dot<double, TPR, U, V, I, true>(indices, a.data, a.x, a.indptr[i], a.indptr[i + 1], lane, ps, pg);
            if constexpr (TPR > 1) acc = group_sum<TPR>(acc, mask);
            v = scale * acc;
            if (lane == 0) sq = fma(v, v, sq);
        }
        // the warp's kWarpRows results to lanes 0..kWarpRows-1, then one coalesced
        // kWarpRows*8-byte segment per rank (lanes spread over the ranks)
        const int src = (wl % kWarpRows) * TPR;
        const double mine = __shfl_sync(kFull, v, src);
        const int64_t row0 = base + (threadIdx.x / 32) * kWarpRows;
        const int64_t r = row0 + (wl % kWarpRows);
        if (r < rows)
            for (int q = wl / kWarpRows; q < a.nparts; q += 32 / kWarpRows) a.y_peers[q][own + r] = mine;
    }
    const double part = block_sum(sq, s_warp);
    __shared__ bool s_last;
    if (threadIdx.x == 0) {
        a.partials[blockIdx.x] = part;
        __threadfence_system();
        s_last = (atomicAdd(a.ticket, 1u) == gridDim.x - 1);
    }
    __syncthreads();
    if (s_last && threadIdx.x < 32) {
        __threadfence_system();
        // every CTA set its error bit (if any) before its ticket: this read sees it
        const bool failed = ld_err(a.err) != 0u;
        if (!failed) {
            double v = 0.0;
            for (unsigned i = threadIdx.x; i < gridDim.x; i += 32) v += __ldcg(&a.partials[i]);
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(kFull, v, off);  // every lane: the total
            if (threadIdx.x < a.nparts) a.y_peers[threadIdx.x][own + a.stride - 1] = v;
            __threadfence_system();
            __syncwarp();
            if (threadIdx.x < a.nparts) st_release_sys(&a.flag_peers[threadIdx.x][a.rank], a.epoch);
        }
        if (threadIdx.x == 0) *a.ticket = 0u;
    }
}

// Bounded wait (2 s) until every rank's flag reached `epoch` (the last iteration's
// pushes have all landed); bit 4 of *err on timeout, and no wait at all when *err is
// already set.
__global__ void p2p_wait_kernel(const unsigned long long* flag_local, int nparts, unsigned long long epoch,
                                uint32_t* err) {
    if (wait_flags(flag_local, nparts, epoch, err)) __threadfence_system();
}

// slot <- sum(shard[0..rows)^2), same deterministic reduction.
__global__ void shard_norm2_kernel(double* shard, int64_t rows, int64_t stride, double* partials, unsigned* ticket) {
    __shared__ double s_warp[32];
    double sq = 0.0;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < rows; i += (int64_t)gridDim.x * blockDim.x)
        sq = fma(shard[i], shard[i], sq);
    const double part = block_sum(sq, s_warp);
    grid_sum_last(part, partials, ticket, shard + stride - 1);
}

// x_out[i] = x~[part*stride + i] / sqrt(sum slots), lambda = sqrt(sum slots).
__global__ void power_finalize_kernel(const double* x, int nparts, int64_t stride, int part, int64_t rows,
                                      double* x_out, double* lambda_out) {
    double t = 0.0;
    for (int r = 0; r < nparts; ++r) t += x[(int64_t)r * stride + stride - 1];
    const double nrm = sqrt(t);
    const double inv = nrm > 0.0 ? 1.0 / nrm : 0.0;
    const double* src = x + (int64_t)part * stride;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < rows; i += (int64_t)gridDim.x * blockDim.x)
        x_out[i] = src[i] * inv;
    if (blockIdx.x == 0 && threadIdx.x == 0 && lambda_out) *lambda_out = nrm;
}

namespace {

constexpr int kPowerMaxGrid = 148 * 16;

struct PowerWs {
    double* partials;
    unsigned* ticket;
};

size_t power_ws_bytes_impl() { return sizeof(double) * kPowerMaxGrid + 256; }

// error word of the fused-exchange path: inside the norm region, after the ticket
uint32_t* p2p_err_word(void* ws) {
    return reinterpret_cast<uint32_t*>(static_cast<char*>(ws) + sizeof(double) * kPowerMaxGrid + 8);
}

PowerWs carve(void* ws) {
    PowerWs w;
    w.partials = static_cast<double*>(ws);
    w.ticket = reinterpret_cast<unsigned*>(static_cast<char*>(ws) + sizeof(double) * kPowerMaxGrid);
    return w;
}

template <int TPR, int U, int V>
void launch_power(const PowerArgs& a, bool i32, int blocks, int threads, cudaStream_t st) {
    if (i32)
        power_step_kernel<TPR, U, V, int32_t><<<blocks, threads, 0, st>>>(a);
    else
        power_step_kernel<TPR, U, V, int64_t><<<blocks, threads, 0, st>>>(a);
}

template <int TPR, int U>
bool power_v(int v, const PowerArgs& a, bool i32, int bl, int th, cudaStream_t st) {
    switch (v) {
        case 1: launch_power<TPR, U, 1>(a, i32, bl, th, st); return true;
        case 2: launch_power<TPR, U, 2>(a, i32, bl, th, st); return true;
        case 4: launch_power<TPR, U, 4>(a, i32, bl, th, st); return true;
    }
    return false;
}

template <int TPR>
bool power_u(int u, int v, const PowerArgs& a, bool i32, int bl, int th, cudaStream_t st) {
    switch (u) {
        case 1: return power_v<TPR, 1>(v, a, i32, bl, th, st);
        case 2: return power_v<TPR, 2>(v, a, i32, bl, th, st);
        case 4: return power_v<TPR, 4>(v, a, i32, bl, th, st);
    }
    return false;
}

bool power_dispatch(int tpr, int u, int v, const PowerArgs& a, bool i32, int bl, int th, cudaStream_t st) {
    switch (tpr) {
        case 4: return power_u<4>(u, v, a, i32, bl, th, st);
        case 8: return power_u<8>(u, v, a, i32, bl, th, st);
        case 16: return power_u<16>(u, v, a, i32, bl, th, st);
        case 32: return power_u<32>(u, v, a, i32, bl, th, st);
    }
    return false;
}

// TG_FLAG_INDEX32: A.indices holds int32 column indices (the padded layout has fewer than
// 2^31 entries); pairs of them need 8-byte alignment, quads (V = 4) 16.
bool index32(const tg_sched& s) { return (s.flags & TG_FLAG_INDEX32) != 0; }

bool stream_aligned(const tg_csr& A, bool i32, int v) {
    const uintptr_t ia = reinterpret_cast<uintptr_t>(A.indices);
    const uintptr_t need = (i32 && v < 4) ? 7u : 15u;
    return ((ia & need) | (reinterpret_cast<uintptr_t>(A.data) & 15u)) == 0;
}

}  // namespace

// stream split (tg_stream.cu)
template <typename T, int MODE>
int stream_run(const tg_csr& A, const T* x, T* y, const T* w, T alpha, T beta, int nparts, int64_t stride,
               const tg_sched& s, void* ws, size_t ws_bytes, cudaStream_t st);
size_t stream_ws_bytes(int64_t nnz, const tg_sched& s, size_t elem);

// Workspace: [norm region: per-CTA partials + ticket | stream plan region].  The two
// regions are disjoint so the slot reduction of tg_shard_norm2_f64 (run when a new x0
// is loaded) never touches the partition table a reused stream plan reads.
static size_t norm_region_bytes() { return (power_ws_bytes_impl() + 255) & ~size_t(255); }

size_t power_ws_bytes(int64_t nnz, const tg_sched& s) {
    size_t b = norm_region_bytes();
    if (s.split == TG_SPLIT_STREAM && nnz > 0) b += stream_ws_bytes(nnz, s, sizeof(double));
    return b;
}

int power_rows_run(const tg_csr& A, int64_t row0, int64_t row1, const double* x, int nparts, int64_t stride,
                   double* y, double* slot_out, const tg_sched& s, void* ws, cudaStream_t st);

int power_step_run(const tg_csr& A, const double* x, int nparts, int64_t stride, double* y, const tg_sched& s,
                   void* ws, size_t ws_bytes, cudaStream_t st) {
    if (nparts < 1 || stride < A.rows + 1)
        return set_error(TG_EINVAL, "power step: need nparts >= 1 and stride >= rows + 1 (nparts=%d stride=%lld)",
                         nparts, (long long)stride);
    const bool i32 = index32(s);
    if (s.split == TG_SPLIT_STREAM && i32)
        return set_error(TG_EUNSUPPORTED, "power step: 32-bit column indices need the rowwise split");
    if (s.split == TG_SPLIT_STREAM && A.nnz > 0 &&
        ((reinterpret_cast<uintptr_t>(A.indices) | reinterpret_cast<uintptr_t>(A.data) |
          reinterpret_cast<uintptr_t>(A.indptr)) & 15u) == 0)
    {
        if (ws == nullptr || ws_bytes < norm_region_bytes())
            return set_error(TG_ENOMEM, "power step: workspace smaller than its norm region");
        return stream_run<double, 2>(A, x, y, nullptr, 0.0, 0.0, nparts, stride, s,
                                     static_cast<char*>(ws) + norm_region_bytes(), ws_bytes - norm_region_bytes(), st);
    }
    if (ws == nullptr || ws_bytes < power_ws_bytes_impl())
        return set_error(TG_ENOMEM, "power step needs %zu workspace bytes, got %zu", power_ws_bytes_impl(), ws_bytes);
    return power_rows_run(A, 0, A.rows, x, nparts, stride, y, y + stride - 1, s, ws, st);
}

// Rows [row0, row1) of the shard A (its indptr is absolute into indices/data), written to
// y[row0, row1), sum of their squares to *slot_out; the rowwise power-step kernel.
int power_rows_run(const tg_csr& A, int64_t row0, int64_t row1, const double* x, int nparts, int64_t stride,
                   double* y, double* slot_out, const tg_sched& s, void* ws, cudaStream_t st) {
    const bool i32 = index32(s);
    const int tpr = s.threads_per_row < 4 ? 4 : s.threads_per_row;
    const int u = s.unroll >= 4 ? 4 : (s.unroll >= 2 ? 2 : 1);
    int v = s.vector_width;
    while (v > 1 && !stream_aligned(A, i32, v)) v /= 2;
    const int threads = s.block_size;
    PowerWs w = carve(ws);
    PowerArgs a{};
    a.indptr = A.indptr + row0;
    a.indices = A.indices;
    a.data = static_cast<const double*>(A.data);
    a.x = x;
    a.nparts = nparts;
    a.stride = stride;
    a.y = y + row0;
    a.rows = row1 - row0;
    a.rows_per_tile = std::max<int64_t>(s.tile, threads / tpr);
    a.partials = w.partials;
    a.ticket = w.ticket;
    a.slot_out = slot_out;
    int64_t blocks = ceil_div(std::max<int64_t>(a.rows, 1), a.rows_per_tile);
    blocks = std::min<int64_t>(blocks, kPowerMaxGrid);
    if (!power_dispatch(tpr, u, v, a, i32, (int)blocks, threads, st))
        return set_error(TG_EUNSUPPORTED, "no power-step instance for TPR=%d U=%d V=%d", tpr, u, v);
    return check_launch("power_step_kernel");
}

template <int TPR, int U, int V>
static void launch_p2p(const PowerP2PArgs& a, bool i32, int blocks, cudaStream_t st) {
    if (i32)
        power_p2p_kernel<TPR, U, V, int32_t><<<blocks, 256, 0, st>>>(a);
    else
        power_p2p_kernel<TPR, U, V, int64_t><<<blocks, 256, 0, st>>>(a);
}

int power_step_p2p_run(const tg_csr& A, const double* x, int nparts, int rank, int64_t stride,
                       double* const* y_peers, unsigned long long* const* flag_peers, unsigned long long epoch,
                       const tg_sched& s, void* ws, size_t ws_bytes, cudaStream_t st) {
    if (nparts < 1 || nparts > 8 || rank < 0 || rank >= nparts || stride < A.rows + 1)
        return set_error(TG_EINVAL, "p2p step: bad nparts/rank/stride (%d, %d, %lld)", nparts, rank, (long long)stride);
    if (epoch < 1) return set_error(TG_EINVAL, "p2p step: epoch must be >= 1");
    if (ws == nullptr || ws_bytes < power_ws_bytes_impl())
        return set_error(TG_ENOMEM, "p2p step needs %zu workspace bytes", power_ws_bytes_impl());
    PowerWs w = carve(ws);
    PowerP2PArgs a{};
    a.indptr = A.indptr;
    a.indices = A.indices;
    a.data = static_cast<const double*>(A.data);
    a.x = x;
    a.nparts = nparts;
    a.rank = rank;
    a.stride = stride;
    for (int q = 0; q < nparts; ++q) {
        if (!y_peers[q] || !flag_peers[q]) return set_error(TG_EINVAL, "p2p step: null peer pointer %d", q);
        a.y_peers[q] = y_peers[q];
        a.flag_peers[q] = flag_peers[q];
    }
    a.flag_local = flag_peers[rank];
    a.epoch = epoch;
    a.rows = A.rows;
    a.partials = w.partials;
    a.ticket = w.ticket;
    a.err = p2p_err_word(ws);
    const int tpr = s.threads_per_row <= 4 ? 4 : 8;
    const int u = s.unroll >= 2 ? 2 : 1;
    const bool i32 = index32(s);
    int v = s.vector_width >= 4 ? 4 : (s.vector_width >= 2 ? 2 : 1);
    while (v > 1 && !stream_aligned(A, i32, v)) v /= 2;
    const int bl = (int)std::min<int64_t>(ceil_div(std::max<int64_t>(A.rows, 1), 256 / tpr), kPowerMaxGrid);
    if (tpr == 4) {
        if (u == 2) {
            if (v == 4) launch_p2p<4, 2, 4>(a, i32, bl, st);
            else if (v == 2) launch_p2p<4, 2, 2>(a, i32, bl, st);
            else launch_p2p<4, 2, 1>(a, i32, bl, st);
        } else {
            if (v == 4) launch_p2p<4, 1, 4>(a, i32, bl, st);
            else if (v == 2) launch_p2p<4, 1, 2>(a, i32, bl, st);
            else launch_p2p<4, 1, 1>(a, i32, bl, st);
        }
    } else {
        if (u == 2) { if (v >= 2) launch_p2p<8, 2, 2>(a, i32, bl, st); else launch_p2p<8, 2, 1>(a, i32, bl, st); }
        else { if (v >= 2) launch_p2p<8, 1, 2>(a, i32, bl, st); else launch_p2p<8, 1, 1>(a, i32, bl, st); }
    }
    return check_launch("power_p2p_kernel");
}

size_t power_err_offset() { return sizeof(double) * kPowerMaxGrid + 8; }

// ------------------------------------------------------------- copy-engine exchange
// The exchange as copies instead of stores from the computing warps: the power step writes
// this rank's rows (and slot) into its own next-iterate buffer; copies (copy engines, over
// NVLink) move them into every peer's buffer, one side stream per peer, joined back into
// the caller's stream; then a one-warp kernel release-stores `epoch` into every rank's
// flag array.  Each step first waits (bounded) for the previous epoch, so it reads a
// complete iterate and nobody overwrites a buffer that is still being read.  Kernels on
// one GPU never wait for one another: the wait is for flags other GPUs release, and the
// release of this GPU comes after its copies in stream order.
struct FlagArgs {
    unsigned long long* f[8];
    int nparts;
    int rank;
    unsigned long long epoch;
};

__global__ void p2p_release_kernel(FlagArgs a) {
    __threadfence_system();
    if ((int)threadIdx.x < a.nparts) st_release_sys(&a.f[threadIdx.x][a.rank], a.epoch);
}

namespace {

struct SideStreams {
    bool ready = false;
    cudaStream_t s[8] = {};
    cudaEvent_t fork = nullptr;
    cudaEvent_t join[8] = {};
};
std::mutex g_side_mu;
std::vector<SideStreams> g_side;  // per device, created on first use, kept for the process

int side_streams(SideStreams** out) {
    int dev = 0;
    int rc = check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
    if (rc != TG_OK) return rc;
    std::lock_guard<std::mutex> lk(g_side_mu);
    if ((int)g_side.size() <= dev) g_side.resize(dev + 1);
    SideStreams& ss = g_side[dev];
    if (!ss.ready) {
        rc = check_cuda(cudaEventCreateWithFlags(&ss.fork, cudaEventDisableTiming), "cudaEventCreate");
        for (int k = 0; k < 8 && rc == TG_OK; ++k) {
            rc = check_cuda(cudaStreamCreateWithFlags(&ss.s[k], cudaStreamNonBlocking), "cudaStreamCreate");
            if (rc == TG_OK) rc = check_cuda(cudaEventCreateWithFlags(&ss.join[k], cudaEventDisableTiming), "cudaEventCreate");
        }
        if (rc != TG_OK) return rc;
        ss.ready = true;
    }
    *out = &ss;
    return TG_OK;
}

}  // namespace

// slot <- parts[0] + parts[1] + ... in that order (the chunks' sums of squares).
__global__ void slot_combine_kernel(const double* parts, int n, double* slot) {
    double t = 0.0;
    for (int k = 0; k < n; ++k) t += parts[k];
    *slot = t;
}

constexpr int kMaxChunks = 16;

// chunk partial slots: inside the norm region, after the ticket and the error word
double* chunk_slots(void* ws) {
    return reinterpret_cast<double*>(static_cast<char*>(ws) + sizeof(double) * kPowerMaxGrid + 64);
}

int p2p_wait_run(const unsigned long long* flag_local, int nparts, unsigned long long epoch, void* ws,
                 size_t ws_bytes, cudaStream_t st);

// One iteration with the copy-engine exchange, pipelined over `nchunks` row chunks:
// wait (bounded) until every rank delivered epoch-1; for each chunk, the power-step kernel
// on its rows, then one copy of those rows to every peer on that peer's side stream, so
// the copies of chunk k run while chunk k+1 computes; the chunks' sums of squares are
// combined in chunk order into the slot, which travels with the last chunk; the copies are
// joined back into `st` and `epoch` is released to every rank.
int power_step_ce_run(const tg_csr& A, const double* x, int nparts, int rank, int64_t stride, double* const* y_peers,
                      unsigned long long* const* flag_peers, unsigned long long epoch, int nchunks, const tg_sched& s,
                      void* ws, size_t ws_bytes, cudaStream_t st) {
    if (nparts < 1 || nparts > 8 || rank < 0 || rank >= nparts || stride < A.rows + 1 || epoch < 1)
        return set_error(TG_EINVAL, "ce step: bad nparts/rank/stride/epoch (%d, %d, %lld)", nparts, rank,
                         (long long)stride);
    if (nchunks < 1 || nchunks > kMaxChunks)
        return set_error(TG_EINVAL, "ce step: nchunks must be in [1, %d] (got %d)", kMaxChunks, nchunks);
    if (s.split == TG_SPLIT_STREAM) return set_error(TG_EUNSUPPORTED, "ce step: the rowwise split only");
    if (ws == nullptr || ws_bytes < power_ws_bytes_impl())
        return set_error(TG_ENOMEM, "ce step needs %zu workspace bytes", power_ws_bytes_impl());
    FlagArgs fa{};
    for (int q = 0; q < nparts; ++q) {
        if (!y_peers[q] || !flag_peers[q]) return set_error(TG_EINVAL, "ce step: null peer pointer %d", q);
        fa.f[q] = flag_peers[q];
    }
    fa.nparts = nparts;
    fa.rank = rank;
    fa.epoch = epoch;
    int rc = TG_OK;
    if (epoch > 1) rc = p2p_wait_run(flag_peers[rank], nparts, epoch - 1, ws, ws_bytes, st);
    if (rc != TG_OK) return rc;
    SideStreams* ss = nullptr;
    if (nparts > 1) {
        rc = side_streams(&ss);
        if (rc != TG_OK) return rc;
    }
    double* own = y_peers[rank] + (int64_t)rank * stride;
    double* parts = chunk_slots(ws);
    for (int k = 0; k < nchunks && rc == TG_OK; ++k) {
        const int64_t r0 = A.rows * k / nchunks, r1 = A.rows * (k + 1) / nchunks;
        rc = power_rows_run(A, r0, r1, x, nparts, stride, own, parts + k, s, ws, st);
        const bool last = k == nchunks - 1;
        if (rc == TG_OK && last) {
            slot_combine_kernel<<<1, 1, 0, st>>>(parts, nchunks, own + stride - 1);
            rc = check_launch("slot_combine_kernel");
        }
        if (rc != TG_OK || nparts == 1) continue;
        const int64_t c0 = r0, c1 = last ? stride : r1;  // the last chunk carries the padding and the slot
        if (c1 <= c0) continue;
        rc = check_cuda(cudaEventRecord(ss->fork, st), "cudaEventRecord");
        int j = 0;
        for (int q = 0; q < nparts && rc == TG_OK; ++q) {
            if (q == rank) continue;
            rc = check_cuda(cudaStreamWaitEvent(ss->s[j], ss->fork, 0), "cudaStreamWaitEvent");
            if (rc == TG_OK)
                rc = check_cuda(cudaMemcpyAsync(y_peers[q] + (int64_t)rank * stride + c0, own + c0,
                                                sizeof(double) * (c1 - c0), cudaMemcpyDefault, ss->s[j]),
                                "cudaMemcpyAsync(peer rows)");
            ++j;
        }
    }
    if (rc != TG_OK) return rc;
    if (nparts > 1) {
        int j = 0;
        for (int q = 0; q < nparts && rc == TG_OK; ++q) {
            if (q == rank) continue;
            rc = check_cuda(cudaEventRecord(ss->join[j], ss->s[j]), "cudaEventRecord");
            if (rc == TG_OK) rc = check_cuda(cudaStreamWaitEvent(st, ss->join[j], 0), "cudaStreamWaitEvent");
            ++j;
        }
        if (rc != TG_OK) return rc;
    }
    p2p_release_kernel<<<1, 32, 0, st>>>(fa);
    return check_launch("p2p_release_kernel");
}

int p2p_wait_run(const unsigned long long* flag_local, int nparts, unsigned long long epoch, void* ws,
                 size_t ws_bytes, cudaStream_t st) {
    if (!flag_local || nparts < 1 || nparts > 8) return set_error(TG_EINVAL, "p2p wait: bad arguments");
    if (ws == nullptr || ws_bytes < power_ws_bytes_impl())
        return set_error(TG_ENOMEM, "p2p wait needs %zu workspace bytes", power_ws_bytes_impl());
    p2p_wait_kernel<<<1, 1, 0, st>>>(flag_local, nparts, epoch, p2p_err_word(ws));
    return check_launch("p2p_wait_kernel");
}

int shard_norm2_run(double* shard, int64_t rows, int64_t stride, void* ws, size_t ws_bytes, cudaStream_t st) {
    if (ws == nullptr || ws_bytes < power_ws_bytes_impl())
        return set_error(TG_ENOMEM, "shard norm needs %zu workspace bytes, got %zu", power_ws_bytes_impl(), ws_bytes);
    PowerWs w = carve(ws);
    int64_t blocks = std::min<int64_t>(std::max<int64_t>(ceil_div(rows, 256), 1), kPowerMaxGrid);
    shard_norm2_kernel<<<(unsigned)blocks, 256, 0, st>>>(shard, rows, stride, w.partials, w.ticket);
    return check_launch("shard_norm2_kernel");
}

int power_finalize_run(const double* x, int nparts, int64_t stride, int part, int64_t rows, double* x_out,
                       double* lambda_out, cudaStream_t st) {
    int64_t blocks = std::min<int64_t>(std::max<int64_t>(ceil_div(rows, 256), 1), 148 * 8);
    power_finalize_kernel<<<(unsigned)blocks, 256, 0, st>>>(x, nparts, stride, part, rows, x_out, lambda_out);
    return check_launch("power_finalize_kernel");
}

}  // namespace tg
