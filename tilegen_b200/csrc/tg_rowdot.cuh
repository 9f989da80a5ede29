// Row dot product of the rowwise split, shared by SpMV (tg_spmv.cu) and the power
// iteration (tg_power.cu): TPR lanes of a group stride over the row, each lane keeps U
// vector loads of V nonzeros in flight (indices/values streamed with an L2 evict_first
// policy, x gathered with evict_last), with a scalar peel to the V-element boundary and
// a ragged scalar tail.
#pragma once

#include "tg_common.cuh"

namespace tg {

// V column indices (int64, or int32 where a caller stored them narrower) and V values
// starting at a V-element boundary.
template <typename T, typename I, int V>
__device__ __forceinline__ void ld_stream_vec(const I* pi, const T* pv, uint64_t pol, int64_t (&c)[V], T (&v)[V]) {
    if constexpr (V == 1) {
        c[0] = ld_stream(pi, pol);
        v[0] = ld_stream(pv, pol);
    } else {
        if constexpr (sizeof(I) == 4 && V == 4) {  // four 32-bit indices in one 16-byte load
            int32_t a, b, d, e;
            ld_stream4(pi, pol, a, b, d, e);
            c[0] = a;
            c[1] = b;
            c[2] = d;
            c[3] = e;
        } else {
#pragma unroll
            for (int e = 0; e < V; e += 2) {
                I a, b;
                ld_stream2(pi + e, pol, a, b);
                c[e] = a;
                c[e + 1] = b;
            }
        }
#pragma unroll
        for (int e = 0; e < V; e += 2) ld_stream2(pv + e, pol, v[e], v[e + 1]);
    }
}

// x gather of row_dot: through L1 (default), or without allocating there (NA).
template <bool NA, typename T>
__device__ __forceinline__ T gather_x(const T* p, uint64_t pol) {
    if constexpr (NA && sizeof(T) == 8) {
        return ld_gather_na(p, pol);
    } else {
        return ld_gather(p, pol);
    }
}

// Dot product of row [p, pe) with x by the TPR lanes of one group (this lane's share).
// I is the column index type (int64_t, or int32_t for a matrix the caller renumbered to
// 32-bit indices); NA gathers x without L1 allocation (the power steps, whose x is 8M
// doubles: measured 0.6 % faster there, 3.5 % slower on a 100k-column SpMV).
template <typename T, int TPR, int U, int V, typename I = int64_t, bool NA = false>
__device__ __forceinline__ T row_dot(const I* __restrict__ idx, const T* __restrict__ val,
                                     const T* __restrict__ x, int64_t p, int64_t pe, int lane, uint64_t ps,
                                     uint64_t pg) {
    Sum<T> acc;
    if constexpr (V == 1) {
        int64_t q = p + lane;
        for (; q + (int64_t)(U - 1) * TPR < pe; q += (int64_t)TPR * U) {
            int64_t c[U];
            T v[U];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                c[u] = (int64_t)ld_stream(idx + q + u * TPR, ps);
                v[u] = ld_stream(val + q + u * TPR, ps);
            }
#pragma unroll
            for (int u = 0; u < U; ++u) acc.mad(v[u], gather_x<NA>(x + c[u], pg));
        }
        for (; q < pe; q += TPR) acc.mad(ld_stream(val + q, ps), gather_x<NA>(x + ld_stream(idx + q, ps), pg));
    } else {
        // peel to a V-element boundary, full vectors, then the ragged tail
        int64_t pa = (p + V - 1) / V * V;
        if (pa > pe) pa = pe;
        for (int64_t q = p + lane; q < pa; q += TPR)
            acc.mad(ld_stream(val + q, ps), gather_x<NA>(x + ld_stream(idx + q, ps), pg));
        const int64_t nv = (pe - pa) / V;
        int64_t k = lane;
        for (; k + (int64_t)(U - 1) * TPR < nv; k += (int64_t)TPR * U) {
            int64_t c[U][V];
            T v[U][V];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int64_t q = pa + (k + (int64_t)u * TPR) * V;
                ld_stream_vec<T, I, V>(idx + q, val + q, ps, c[u], v[u]);
            }
#pragma unroll
            for (int u = 0; u < U; ++u)
#pragma unroll
                for (int e = 0; e < V; ++e) acc.mad(v[u][e], gather_x<NA>(x + c[u][e], pg));
        }
        for (; k < nv; k += TPR) {
            int64_t c[V];
            T v[V];
            const int64_t q = pa + k * V;
            ld_stream_vec<T, I, V>(idx + q, val + q, ps, c, v);
#pragma unroll
            for (int e = 0; e < V; ++e) acc.mad(v[e], gather_x<NA>(x + c[e], pg));
        }
        for (int64_t q = pa + nv * V + lane; q < pe; q += TPR)
            acc.mad(ld_stream(val + q, ps), gather_x<NA>(x + ld_stream(idx + q, ps), pg));
    }
    return acc.get();
}

}  // namespace tg
