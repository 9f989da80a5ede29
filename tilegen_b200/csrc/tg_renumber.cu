// tg_renumber_columns: column renumbering of a row shard to the padded iterate layout of
// the power iteration (the device half of the nnz-balanced partitioner).
//
// With the rows split at bounds[0] = 0 < bounds[1] < ... < bounds[P] = N and every shard
// stored at a stride of `stride` doubles, column j (owned by shard q: bounds[q] <= j <
// bounds[q+1]) moves to q * stride + (j - bounds[q]).  One streaming pass, HBM-bound
// (16 bytes per nonzero); the bounds travel in the kernel parameters.
#include <algorithm>

#include "tg_common.cuh"

namespace tg {
namespace {

constexpr int kMaxParts = 64;

struct Bounds {
    int64_t b[kMaxParts + 1];
    int parts;
};

// OUT = int64_t, or int32_t when the padded layout has fewer than 2^31 entries (the
// narrower indices cut the SpMV's CSR stream from 16 to 12 bytes per nonzero).
template <typename OUT>
__global__ void __launch_bounds__(256) renumber_kernel(const int64_t* __restrict__ in, OUT* out, int64_t n,
                                                       const Bounds bd, int64_t stride) {
    const uint64_t ps = policy_evict_first();
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t j = ld_stream(in + i, ps);
        int q = 0;
        while (q + 1 < bd.parts && j >= bd.b[q + 1]) ++q;  // parts <= 64: a short scan
        out[i] = (OUT)((int64_t)q * stride + (j - bd.b[q]));
    }
}

template <typename OUT>
int renumber_run(const int64_t* indices, OUT* out, int64_t nnz, const int64_t* bounds, int32_t nparts,
                 int64_t stride, tg_stream_t stream, const char* op) {
    if (nnz < 0 || nparts < 1 || nparts > kMaxParts || stride < 1)
        return set_error(TG_EINVAL, "%s: bad arguments (nnz=%lld nparts=%d stride=%lld)", op, (long long)nnz, nparts,
                         (long long)stride);
    if (!bounds || (nnz > 0 && (!indices || !out))) return set_error(TG_EINVAL, "%s: null pointer argument", op);
    if (sizeof(OUT) == 4 && (int64_t)nparts * stride > INT32_MAX)
        return set_error(TG_EINVAL, "%s: the padded layout (%lld entries) does not fit 32-bit indices", op,
                         (long long)((int64_t)nparts * stride));
    Bounds bd{};
    bd.parts = nparts;
    for (int q = 0; q <= nparts; ++q) {
        bd.b[q] = bounds[q];
        if (q > 0 && (bd.b[q] < bd.b[q - 1] || bd.b[q] - bd.b[q - 1] > stride - 1))
            return set_error(TG_EINVAL, "%s: bounds must be non-decreasing with shards < stride", op);
    }
    if (bd.b[0] != 0) return set_error(TG_EINVAL, "%s: bounds[0] must be 0", op);
    if (nnz == 0) return TG_OK;
    const int64_t blocks = std::min<int64_t>(ceil_div(nnz, 256), 148 * 16);
    renumber_kernel<OUT><<<(unsigned)blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(indices, out, nnz, bd,
                                                                                         stride);
    return check_launch("renumber_kernel");
}

}  // namespace
}  // namespace tg

using namespace tg;

extern "C" int tg_renumber_columns_i32(const int64_t* indices, int32_t* out, int64_t nnz, const int64_t* bounds,
                                       int32_t nparts, int64_t stride, tg_stream_t stream) {
    return renumber_run<int32_t>(indices, out, nnz, bounds, nparts, stride, stream, "tg_renumber_columns_i32");
}

extern "C" int tg_renumber_columns(const int64_t* indices, int64_t* out, int64_t nnz, const int64_t* bounds,
                                   int32_t nparts, int64_t stride, tg_stream_t stream) {
    return renumber_run<int64_t>(indices, out, nnz, bounds, nparts, stride, stream, "tg_renumber_columns");
}

