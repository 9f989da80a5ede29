// Shared device helpers for the sm_100a sparse kernels of libtilegen_b200.so.
//
// * cache-policy loads: the CSR stream (indices, values) is read exactly once per call,
//   so it is fetched with an L2 evict_first policy and no L1 allocation; the dense
//   gather operands (x, B, V, U) are fetched with evict_last so that they stay in the
//   126 MB L2 while the stream flows past them.
// * TMA bulk copies (cp.async.bulk, 1-D, no multicast) + mbarrier helpers used to stage
//   nnz chunks into shared memory.
// * error plumbing shared by every translation unit (definitions in tg_abi.cu).
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

#include "../../include/tilegen_b200.h"

namespace tg {

// ------------------------------------------------------------------ host errors
int set_error(int status, const char* fmt, ...);
int check_cuda(cudaError_t e, const char* what);
int check_launch(const char* what);

constexpr int kWarp = 32;
constexpr unsigned kFull = 0xffffffffu;

// ------------------------------------------------------------ device loads
__device__ __forceinline__ uint64_t policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

__device__ __forceinline__ uint64_t policy_evict_last() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// Streamed-once loads (CSR indices / values).
__device__ __forceinline__ int64_t ld_stream(const int64_t* p, uint64_t pol) {
    int64_t v;
    asm("ld.global.nc.L1::no_allocate.L2::cache_hint.s64 %0, [%1], %2;" : "=l"(v) : "l"(p), "l"(pol));
    return v;
}
__device__ __forceinline__ int32_t ld_stream(const int32_t* p, uint64_t pol) {
    int32_t v;
    asm("ld.global.nc.L1::no_allocate.L2::cache_hint.s32 %0, [%1], %2;" : "=r"(v) : "l"(p), "l"(pol));
    return v;
}
__device__ __forceinline__ double ld_stream(const double* p, uint64_t pol) {
    double v;
    asm("ld.global.nc.L1::no_allocate.L2::cache_hint.f64 %0, [%1], %2;" : "=d"(v) : "l"(p), "l"(pol));
    return v;
}
__device__ __forceinline__ float ld_stream(const float* p, uint64_t pol) {
    float v;
    asm("ld.global.nc.L1::no_allocate.L2::cache_hint.f32 %0, [%1], %2;" : "=f"(v) : "l"(p), "l"(pol));
    return v;
}
// Four int32 stream elements in one 16-byte load; the address must be 16-byte aligned.
__device__ __forceinline__ void ld_stream4(const int32_t* p, uint64_t pol, int32_t& a, int32_t& b, int32_t& c,
                                           int32_t& d) {
    asm("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.s32 {%0, %1, %2, %3}, [%4], %5;"
        : "=r"(a), "=r"(b), "=r"(c), "=r"(d) : "l"(p), "l"(pol));
}
// Vector stream loads of two elements; the address must be aligned to their size
// (16 bytes for 64-bit elements, 8 for 32-bit ones).
__device__ __forceinline__ void ld_stream2(const int32_t* p, uint64_t pol, int32_t& a, int32_t& b) {
    asm("ld.global.nc.L1::no_allocate.L2::cache_hint.v2.s32 {%0, %1}, [%2], %3;"
        : "=r"(a), "=r"(b) : "l"(p), "l"(pol));
}
__device__ __forceinline__ void ld_stream2(const int64_t* p, uint64_t pol, int64_t& a, int64_t& b) {
    asm("ld.global.nc.L1::no_allocate.L2::cache_hint.v2.s64 {%0, %1}, [%2], %3;"
        : "=l"(a), "=l"(b) : "l"(p), "l"(pol));
}
__device__ __forceinline__ void ld_stream2(const double* p, uint64_t pol, double& a, double& b) {
    asm("ld.global.nc.L1::no_allocate.L2::cache_hint.v2.f64 {%0, %1}, [%2], %3;"
        : "=d"(a), "=d"(b) : "l"(p), "l"(pol));
}
__device__ __forceinline__ void ld_stream2(const float* p, uint64_t pol, float& a, float& b) {
    asm("ld.global.nc.L1::no_allocate.L2::cache_hint.v2.f32 {%0, %1}, [%2], %3;"
        : "=f"(a), "=f"(b) : "l"(p), "l"(pol));
}

// Gather loads of the dense operand (kept in L2).
__device__ __forceinline__ double ld_gather(const double* p, uint64_t pol) {
    double v;
    asm("ld.global.nc.L2::cache_hint.f64 %0, [%1], %2;" : "=d"(v) : "l"(p), "l"(pol));
    return v;
}
// The same gather without an L1 line: for an operand far larger than L1 whose elements are
// not reused by the same SM (the power iteration's 64 MB iterate), allocating in L1 only
// costs L1 tag work.
__device__ __forceinline__ double ld_gather_na(const double* p, uint64_t pol) {
    double v;
    asm("ld.global.nc.L1::no_allocate.L2::cache_hint.f64 %0, [%1], %2;" : "=d"(v) : "l"(p), "l"(pol));
    return v;
}
__device__ __forceinline__ float ld_gather(const float* p, uint64_t pol) {
    float v;
    asm("ld.global.nc.L2::cache_hint.f32 %0, [%1], %2;" : "=f"(v) : "l"(p), "l"(pol));
    return v;
}

// Vector of VEC elements of T, used for row slices of the dense operands of SpMM/SDDMM.
template <typename T, int VEC>
struct Vec {
    T v[VEC];
};

template <typename T, int VEC>
__device__ __forceinline__ Vec<T, VEC> ld_gather_vec(const T* p, uint64_t pol) {
    Vec<T, VEC> r;
    if constexpr (VEC == 1) {
        r.v[0] = ld_gather(p, pol);
    } else if constexpr (sizeof(T) == 4 && VEC == 4) {
        asm("ld.global.nc.L2::cache_hint.v4.f32 {%0, %1, %2, %3}, [%4], %5;"
            : "=f"(r.v[0]), "=f"(r.v[1]), "=f"(r.v[2]), "=f"(r.v[3]) : "l"(p), "l"(pol));
    } else if constexpr (sizeof(T) == 4 && VEC == 2) {
        asm("ld.global.nc.L2::cache_hint.v2.f32 {%0, %1}, [%2], %3;"
            : "=f"(r.v[0]), "=f"(r.v[1]) : "l"(p), "l"(pol));
    } else if constexpr (sizeof(T) == 8 && VEC == 2) {
        asm("ld.global.nc.L2::cache_hint.v2.f64 {%0, %1}, [%2], %3;"
            : "=d"(r.v[0]), "=d"(r.v[1]) : "l"(p), "l"(pol));
    } else {
#pragma unroll
        for (int i = 0; i < VEC; ++i) r.v[i] = ld_gather(p + i, pol);
    }
    return r;
}

template <typename T, int VEC>
__device__ __forceinline__ void st_vec(T* p, const Vec<T, VEC>& r) {
    if constexpr (sizeof(T) == 4 && VEC == 4) {
        *reinterpret_cast<float4*>(p) = make_float4(r.v[0], r.v[1], r.v[2], r.v[3]);
    } else if constexpr (sizeof(T) == 4 && VEC == 2) {
        *reinterpret_cast<float2*>(p) = make_float2(r.v[0], r.v[1]);
    } else if constexpr (sizeof(T) == 8 && VEC == 2) {
        *reinterpret_cast<double2*>(p) = make_double2(r.v[0], r.v[1]);
    } else {
#pragma unroll
        for (int i = 0; i < VEC; ++i) p[i] = r.v[i];
    }
}

// L2-coherent load used by the last-arriving contributor of a split row to read the
// partial sums other CTAs published (bypasses L1, which is not coherent across SMs).
template <typename T>
__device__ __forceinline__ T ld_cg(const T* p) {
    return __ldcg(p);
}

// Sum of the partials p[0], p[stride], ..., p[(n-1)*stride] added in index order into s.
// The loads are issued eight at a time (independent, all in flight together) and the
// adds stay in order, so the result is the same as the one-at-a-time loop but the
// latency is paid once per eight partials instead of once per partial.
template <typename T, class SUM>
__device__ __forceinline__ void add_partials(SUM& s, const T* p, int64_t n, int64_t stride) {
    int64_t c = 0;
    for (; c + 8 <= n; c += 8) {
        T v[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) v[k] = ld_cg(p + (c + k) * stride);
#pragma unroll
        for (int k = 0; k < 8; ++k) s.add(v[k]);
    }
    for (; c < n; ++c) s.add(ld_cg(p + c * stride));
}

// ------------------------------------------------------------ programmatic dependent launch
// A kernel launched with programmatic stream serialisation may start while the kernel
// before it on the stream is still running.  The earlier kernel calls pdl_trigger() to
// let it start; the later one calls pdl_wait() before it reads anything the earlier
// kernel writes (pdl_wait returns once that kernel has completed and its writes are
// visible, and at once when there is no such dependency).
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// ------------------------------------------------------------ TMA bulk copies
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Bounded wait on phase `parity` of the mbarrier.  Returns false once 2 s of wall time
// have passed (the caller records an error and skips the dependent work) instead of
// spinning forever; every copy this library issues completes in microseconds.
__device__ __forceinline__ bool mbar_try(uint32_t a, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(a), "r"(parity)
        : "memory");
    return done != 0;
}

__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
    const uint32_t a = smem_addr(bar);
    if (mbar_try(a, parity)) return true;  // fast path: no timer read
    const uint64_t t0 = globaltimer_ns();
    for (;;) {
        if (mbar_try(a, parity)) return true;
        if (globaltimer_ns() - t0 > 2000000000ull) return false;
    }
}

// Non-blocking check of phase `parity` (mbarrier.test_wait).
__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return done != 0;
}

// 1-D bulk copy global -> shared, completion counted on `bar` (complete_tx bytes).
// Both addresses must be 16-byte aligned and `bytes` a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                         uint64_t pol) {
    asm volatile(
        "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
            smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(pol)
        : "memory");
}

// ------------------------------------------------------------ warp helpers
template <int W, typename T>
__device__ __forceinline__ T group_sum(T v, unsigned mask) {
#pragma unroll
    for (int off = W / 2; off > 0; off >>= 1) v += __shfl_xor_sync(mask, v, off, W);
    return v;
}

// Running sum of products.  fp64 accumulates with fused multiply-adds; fp32 uses
// compensated (Kahan) summation of the rounded products, so a long fp32 row keeps an
// error of a few ulps of the row's magnitude instead of growing with its length.  The
// kernels are HBM-bound, so the three extra adds per term cost no time.
template <typename T>
struct Sum;

template <>
struct Sum<double> {
    double s = 0.0;
    __device__ __forceinline__ void mad(double a, double b) { s = fma(a, b, s); }
    __device__ __forceinline__ void add(double v) { s += v; }
    __device__ __forceinline__ double get() const { return s; }
};

template <>
struct Sum<float> {
    float s = 0.0f, c = 0.0f;
    __device__ __forceinline__ void add(float v) {
        const float y = v - c;
        const float t = s + y;
        c = (t - s) - y;
        s = t;
    }
    __device__ __forceinline__ void mad(float a, float b) { add(a * b); }
    __device__ __forceinline__ float get() const { return s; }
};

// Epilogue of the SpMV family: plain y = acc, or the fused axpy z = alpha*acc + beta*w.
template <typename T, bool AXPY>
struct Epi {
    const T* w;
    T alpha, beta;
    __device__ __forceinline__ T operator()(T acc, int64_t row) const {
        if constexpr (AXPY) {
            return alpha * acc + beta * w[row];
        } else {
            return acc;
        }
    }
};

__host__ __device__ inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

}  // namespace tg
