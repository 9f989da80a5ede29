// tg_gather_probe_f64: the random-gather floor of a CSR SpMV, measured on the device.
//
// A CSR SpMV over uniformly scattered columns is bound by how fast the SMs can gather
// 8-byte x values from random addresses (one 32-byte L2 sector per gather), not by the
// HBM stream of indices and values.  This kernel performs the same gathers as the power
// step's SpMV -- the same column indices, the same load instruction and cache policy
// (ld.global.nc, no L1 allocation, L2 evict_last), four gathers in flight per thread --
// and nothing else (no values, no row offsets, no row reductions, no output vector), so
// the time it takes is the floor for the SpMV's gather traffic on this GPU.  Benchmarks report the SpMV's time
// against it next to the HBM roofline.
//
// tg_row_gather_probe_f32 does the same for the dense-row gathers of a CSR SpMM / SDDMM:
// for every position i < n it reads row indices[i] of a row-major fp32 operand of K = 64
// or 128 columns (one 16-byte vector per lane, K/4 lanes per row, the SpMM kernel's load
// instruction and L2 evict_last policy, four rows in flight per lane group) and adds it
// into a checksum -- no values, no row walk, no accumulator rows, no output matrix.  On an
// operand larger than L2 at random rows, its time is the DRAM floor of those gathers.
//
// A measurement aid only: it is built into its own library (libtg_gather_probe.so, loaded
// by the benchmark), not into libtilegen_b200.so.
//
//   int tg_gather_probe_f64(const int64_t* indices, int64_t n, const double* x, double* out,
//                           void* stream);
//   int tg_gather_probe_i32_f64(const int32_t* indices, ...);   (int32 column indices)
// *out += sum of x[indices[i]], i < n (device pointers; *out zeroed by the caller).
//   int tg_row_gather_probe_f32(const int64_t* indices, int64_t n, const float* B, int64_t K,
//                               double* out, void* stream);
// *out += sum of B[indices[i], :] (B row-major, K columns, 16-byte aligned; *out zeroed by
// the caller).
// Returns 0, -1 for a bad argument, -2 when the launch failed.
#include <algorithm>

#include "../csrc/tg_common.cuh"

namespace tg {
namespace {

template <typename I>
__global__ void __launch_bounds__(256) gather_probe_kernel(const I* __restrict__ idx, int64_t n,
                                                           const double* __restrict__ x, double* out) {
    const uint64_t ps = policy_evict_first();
    const uint64_t pg = policy_evict_last();
    const int64_t T = (int64_t)gridDim.x * blockDim.x;
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    double acc = 0.0;
    for (; i + 3 * T < n; i += 4 * T) {
        const int64_t c0 = ld_stream(idx + i, ps), c1 = ld_stream(idx + i + T, ps);
        const int64_t c2 = ld_stream(idx + i + 2 * T, ps), c3 = ld_stream(idx + i + 3 * T, ps);
        const double g0 = ld_gather_na(x + c0, pg), g1 = ld_gather_na(x + c1, pg);
        const double g2 = ld_gather_na(x + c2, pg), g3 = ld_gather_na(x + c3, pg);
        acc += (g0 + g1) + (g2 + g3);
    }
    for (; i < n; i += T) acc += ld_gather_na(x + ld_stream(idx + i, ps), pg);
    acc = group_sum<kWarp>(acc, kFull);
    if ((threadIdx.x % kWarp) == 0) atomicAdd(out, acc);
}

template <typename I>
int probe_run(const I* indices, int64_t n, const double* x, double* out, void* stream) {
    if (n < 0) return TG_EINVAL;
    if (n > 0 && (!indices || !x || !out)) return TG_EINVAL;
    if (n == 0) return TG_OK;
    const int64_t blocks = std::min<int64_t>(ceil_div(n, 256 * 4), 148 * 16);
    gather_probe_kernel<I><<<(unsigned)blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(indices, n, x, out);
    return cudaGetLastError() == cudaSuccess ? TG_OK : TG_ECUDA;
}

template <int G, int U>
__global__ void __launch_bounds__(256) row_gather_probe_kernel(const int64_t* __restrict__ idx, int64_t n,
                                                               const float* __restrict__ B, int64_t K, double* out) {
    const uint64_t ps = policy_evict_first();
    const uint64_t pg = policy_evict_last();
    const int lane = threadIdx.x % G;
    const int64_t gid = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) / G;
    const int64_t ngroups = ((int64_t)gridDim.x * blockDim.x) / G;
    const int64_t col = (int64_t)lane * 4;
    float acc = 0.0f;
    for (int64_t i0 = gid * U; i0 < n; i0 += ngroups * U) {
        int64_t c[U];
#pragma unroll
        for (int u = 0; u < U; ++u) c[u] = i0 + u < n ? ld_stream(idx + i0 + u, ps) : -1;
        Vec<float, 4> v[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            v[u].v[0] = v[u].v[1] = v[u].v[2] = v[u].v[3] = 0.0f;
            if (c[u] >= 0) v[u] = ld_gather_vec<float, 4>(B + c[u] * K + col, pg);
        }
#pragma unroll
        for (int u = 0; u < U; ++u) acc += (v[u].v[0] + v[u].v[1]) + (v[u].v[2] + v[u].v[3]);
    }
    acc = group_sum<kWarp>(acc, kFull);
    if ((threadIdx.x % kWarp) == 0) atomicAdd(out, (double)acc);
}

int row_probe_run(const int64_t* indices, int64_t n, const float* B, int64_t K, double* out, void* stream) {
    if (n < 0 || (K != 64 && K != 128)) return TG_EINVAL;
    if (n > 0 && (!indices || !B || !out || (reinterpret_cast<uintptr_t>(B) & 15u) != 0)) return TG_EINVAL;
    if (n == 0) return TG_OK;
    const int G = (int)(K / 4);
    const int64_t blocks = std::min<int64_t>(ceil_div(n, (256 / G) * 4), 148 * 16);
    if (G == 32)
        row_gather_probe_kernel<32, 4><<<(unsigned)blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(indices, n, B,
                                                                                                        K, out);
    else
        row_gather_probe_kernel<16, 4><<<(unsigned)blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(indices, n, B,
                                                                                                        K, out);
    return cudaGetLastError() == cudaSuccess ? TG_OK : TG_ECUDA;
}

}  // namespace
}  // namespace tg

using namespace tg;

extern "C" __attribute__((visibility("default"))) int tg_gather_probe_f64(const int64_t* indices, int64_t n,
                                                                         const double* x, double* out, void* stream) {
    return probe_run<int64_t>(indices, n, x, out, stream);
}

// The same with int32 column indices (a matrix renumbered to 32-bit indices).
extern "C" __attribute__((visibility("default"))) int tg_gather_probe_i32_f64(const int32_t* indices, int64_t n,
                                                                             const double* x, double* out,
                                                                             void* stream) {
    return probe_run<int32_t>(indices, n, x, out, stream);
}

// Dense-row gathers of an SpMM / SDDMM (K = 64 or 128 fp32 columns).
extern "C" __attribute__((visibility("default"))) int tg_row_gather_probe_f32(const int64_t* indices, int64_t n,
                                                                             const float* B, int64_t K, double* out,
                                                                             void* stream) {
    return row_probe_run(indices, n, B, K, out, stream);
}
