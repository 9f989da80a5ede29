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

#include "tg_rowdot.cuh"

namespace tg {

struct PowerArgs {
    const int64_t* indptr;
    const int64_t* indices;  // renumbered to the padded layout
    const double* data;
    const double* x;  // padded input iterate, nparts * stride
    int nparts;
    int64_t stride;
    double* y;  // output shard (stride doubles, slot at stride-1)
    int64_t rows;
    int64_t rows_per_tile;
    double* partials;  // [gridDim.x]
    unsigned* ticket;  // [1], zero between launches
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

template <int TPR, int U, int V>
__global__ void __launch_bounds__(1024) power_step_kernel(PowerArgs a) {
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
            double acc = row_dot<double, TPR, U, V>(a.indices, a.data, a.x, a.indptr[i], a.indptr[i + 1], lane, ps, pg);
            if constexpr (TPR > 1) acc = group_sum<TPR>(acc, mask);
            if (lane == 0) {
                const double v = scale * acc;
                a.y[i] = v;
                sq = fma(v, v, sq);
            }
        }
    }
    const double part = block_sum(sq, s_warp);
    grid_sum_last(part, a.partials, a.ticket, a.y + a.stride - 1);
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

PowerWs carve(void* ws) {
    PowerWs w;
    w.partials = static_cast<double*>(ws);
    w.ticket = reinterpret_cast<unsigned*>(static_cast<char*>(ws) + sizeof(double) * kPowerMaxGrid);
    return w;
}

template <int TPR, int U, int V>
void launch_power(const PowerArgs& a, int blocks, int threads, cudaStream_t st) {
    power_step_kernel<TPR, U, V><<<blocks, threads, 0, st>>>(a);
}

template <int TPR, int U>
bool power_v(int v, const PowerArgs& a, int bl, int th, cudaStream_t st) {
    switch (v) {
        case 1: launch_power<TPR, U, 1>(a, bl, th, st); return true;
        case 2: launch_power<TPR, U, 2>(a, bl, th, st); return true;
        case 4: launch_power<TPR, U, 4>(a, bl, th, st); return true;
    }
    return false;
}

template <int TPR>
bool power_u(int u, int v, const PowerArgs& a, int bl, int th, cudaStream_t st) {
    switch (u) {
        case 1: return power_v<TPR, 1>(v, a, bl, th, st);
        case 2: return power_v<TPR, 2>(v, a, bl, th, st);
        case 4: return power_v<TPR, 4>(v, a, bl, th, st);
    }
    return false;
}

bool power_dispatch(int tpr, int u, int v, const PowerArgs& a, int bl, int th, cudaStream_t st) {
    switch (tpr) {
        case 4: return power_u<4>(u, v, a, bl, th, st);
        case 8: return power_u<8>(u, v, a, bl, th, st);
        case 16: return power_u<16>(u, v, a, bl, th, st);
        case 32: return power_u<32>(u, v, a, bl, th, st);
    }
    return false;
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

int power_step_run(const tg_csr& A, const double* x, int nparts, int64_t stride, double* y, const tg_sched& s,
                   void* ws, size_t ws_bytes, cudaStream_t st) {
    if (nparts < 1 || stride < A.rows + 1)
        return set_error(TG_EINVAL, "power step: need nparts >= 1 and stride >= rows + 1 (nparts=%d stride=%lld)",
                         nparts, (long long)stride);
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
    if (nparts < 1 || stride < A.rows + 1)
        return set_error(TG_EINVAL, "power step: need nparts >= 1 and stride >= rows + 1 (nparts=%d stride=%lld)",
                         nparts, (long long)stride);
    const int tpr = s.threads_per_row < 4 ? 4 : s.threads_per_row;
    const int u = s.unroll >= 4 ? 4 : (s.unroll >= 2 ? 2 : 1);
    int v = s.vector_width;
    if ((reinterpret_cast<uintptr_t>(A.indices) | reinterpret_cast<uintptr_t>(A.data)) & 15u) v = 1;
    const int threads = s.block_size;
    PowerWs w = carve(ws);
    PowerArgs a{};
    a.indptr = A.indptr;
    a.indices = A.indices;
    a.data = static_cast<const double*>(A.data);
    a.x = x;
    a.nparts = nparts;
    a.stride = stride;
    a.y = y;
    a.rows = A.rows;
    a.rows_per_tile = std::max<int64_t>(s.tile, threads / tpr);
    a.partials = w.partials;
    a.ticket = w.ticket;
    int64_t blocks = ceil_div(std::max<int64_t>(A.rows, 1), a.rows_per_tile);
    blocks = std::min<int64_t>(blocks, kPowerMaxGrid);
    if (!power_dispatch(tpr, u, v, a, (int)blocks, threads, st))
        return set_error(TG_EUNSUPPORTED, "no power-step instance for TPR=%d U=%d V=%d", tpr, u, v);
    return check_launch("power_step_kernel");
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
