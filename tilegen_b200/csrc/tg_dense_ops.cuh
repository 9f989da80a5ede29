// CSR x dense SpMM and CSR-sampled SDDMM kernels for sm_100a (templates; instantiated
// per value type in tg_spmm_*.cu / tg_sddmm_*.cu).
//
// Reference: SpMM `row_dense_out` templates K4/K5 (tilegen/codegen.py:646-685, math
// cpp/src/ref.cpp:31-43); SDDMM `sparse_out` template K6 (tilegen/codegen.py:688-714,
// math cpp/src/ref.cpp:46-59).
//
// Both ops gather one dense row (B[j,:] or V[j,:]) per nonzero, so the unit of work is a
// GROUP of G lanes that walks nonzeros in order: each lane owns NCV column vectors of
// VEC elements (columns lane*VEC + m*G*VEC), the group keeps U nonzeros' gathers in
// flight, and row changes are found by comparing positions against indptr (a merge of
// row ends and nonzero positions).  Work units are either rows (rowwise split) or
// nnz-balanced chunks of S nonzeros (merge split, tg_split.cuh) so that power-law rows
// are spread over many groups.
//
// SpMM writes C (no pre-zeroing needed); rows split across chunks are reduced with the
// deterministic last-arriver protocol using K-wide partial rows.  SDDMM writes one value
// per nonzero in A's order, so the output pattern is A's by construction.
//
// Column tiling (host side, tg_dense_host.cuh): when the gathered operand (B or V) is
// larger than an L2 budget, the call is split into launches over column tiles whose
// slab of it fits in L2, so each dense row is fetched from DRAM about once instead of
// once per nonzero that touches it; the CSR stream is re-read per tile.
#pragma once

#include "tg_split.cuh"

namespace tg {

template <typename T>
struct DenseArgs {
    const int64_t* indptr;
    const int64_t* indices;
    const T* data;
    const T* B;   // SpMM: B (cols x ld); SDDMM: V (cols x ld)
    const T* U;   // SDDMM: U (rows x ld)
    T* C;         // SpMM: C (rows x ld); SDDMM: out[nnz]
    int64_t rows;
    int64_t nnz;
    int64_t ld;      // row stride of the dense operands (elements)
    int64_t kt;      // columns handled by this launch (tile width, <= G*VEC*NCV)
    int64_t kpart;   // row width of the partial buffers (G*VEC*NCV)
    int64_t S;       // merge: nonzeros per chunk
    int64_t nunits;  // rows (rowwise) or chunks (merge)
    int64_t row_limit;
    int pass;        // SDDMM column tile: kPassOnly / kPassFirst / kPassMid / kPassLast
    const int64_t* own_first;
    int* cnt;
    T* head;
    T* tail;
};

// SDDMM over column tiles.  Each nonzero's dot product is accumulated in out[p] across
// the launches, one tile after the other (a fixed order), and A's value is applied by
// the last one: only tile: out = a * dot; first: out = dot; middle: out += dot; last:
// out = a * (out + dot).
constexpr int kPassOnly = 0, kPassFirst = 1, kPassMid = 2, kPassLast = 3;

template <int G>
__device__ __forceinline__ unsigned group_mask() {
    if constexpr (G == 32) {
        return kFull;
    } else {
        return ((1u << G) - 1u) << ((threadIdx.x % 32) / G * G);
    }
}

// First row of a merge chunk's walk: empty rows starting exactly at cs, else the row
// containing position cs.
__device__ __forceinline__ int64_t chunk_first_row(const int64_t* indptr, const int64_t* own_first, int64_t rows,
                                                   int64_t c, int64_t cs) {
    const int64_t of = own_first[c];
    if (of < rows && indptr[of] == cs) return of;
    return of - 1;
}

// ------------------------------------------------------------------ SpMM
template <typename T, int G, int VEC, int NCV>
struct RowAcc {
    Sum<T> v[NCV][VEC];
    __device__ __forceinline__ void zero() {
#pragma unroll
        for (int m = 0; m < NCV; ++m)
#pragma unroll
            for (int e = 0; e < VEC; ++e) v[m][e] = Sum<T>();
    }
};

template <typename T, int G, int VEC, int NCV>
__device__ __forceinline__ void store_row(T* dst, const RowAcc<T, G, VEC, NCV>& acc, int lane, int64_t kt) {
#pragma unroll
    for (int m = 0; m < NCV; ++m) {
        const int64_t col = ((int64_t)lane + (int64_t)m * G) * VEC;
        if (col < kt) {
            Vec<T, VEC> r;
#pragma unroll
            for (int e = 0; e < VEC; ++e) r.v[e] = acc.v[m][e].get();
            st_vec<T, VEC>(dst + col, r);
        }
    }
}

// Arrival of one group on split row `row` (chunks ca..cb) after storing its partial.
template <typename T, int G, int VEC, int NCV>
__device__ __forceinline__ void split_arrive_rows(const DenseArgs<T>& a, int64_t row, int64_t ca, int64_t cb,
                                                  int lane, unsigned gmask) {
    __threadfence();
    __syncwarp(gmask);
    int old = 0;
    if (lane == 0) old = atomicAdd(&a.cnt[ca], 1);
    old = __shfl_sync(gmask, old, 0, G);
    if (old == (int)(cb - ca)) {
        __threadfence();
#pragma unroll
        for (int m = 0; m < NCV; ++m) {
            const int64_t col0 = ((int64_t)lane + (int64_t)m * G) * VEC;
            if (col0 < a.kt) {
#pragma unroll
                for (int e = 0; e < VEC; ++e) {
                    const int64_t col = col0 + e;
                    Sum<T> s;
                    s.add(ld_cg(&a.tail[ca * a.kpart + col]));
                    add_partials(s, a.head + (ca + 1) * a.kpart + col, cb - ca, a.kpart);
                    if (row < a.row_limit) a.C[row * a.ld + col] = s.get();
                }
            }
        }
        __syncwarp(gmask);
        if (lane == 0) a.cnt[ca] = 0;
    }
}

template <typename T, int G, int VEC, int NCV, int U, bool MERGE>
__global__ void __launch_bounds__(512) spmm_kernel(DenseArgs<T> a) {
    const int lane = threadIdx.x % G;
    const unsigned gmask = group_mask<G>();
    const int64_t gid = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) / G;
    const int64_t ngroups = ((int64_t)gridDim.x * blockDim.x) / G;
    const uint64_t ps = policy_evict_first();
    const uint64_t pg = policy_evict_last();

    for (int64_t unit = gid; unit < a.nunits; unit += ngroups) {
        int64_t cs, ce, r, nxt;
        bool head = false;
        if constexpr (MERGE) {
            cs = unit * a.S;
            ce = min(cs + a.S, a.nnz);
            r = chunk_first_row(a.indptr, a.own_first, a.rows, unit, cs);
            head = a.indptr[r] < cs;
            nxt = a.indptr[r + 1];
        } else {
            r = unit;
            cs = a.indptr[r];
            ce = a.indptr[r + 1];
            nxt = ce;
        }
        bool first = true;
        RowAcc<T, G, VEC, NCV> acc;
        acc.zero();
        for (int64_t q0 = cs; q0 < ce; q0 += U) {
            int64_t cidx[U];
            T cval[U];
            Vec<T, VEC> b[U][NCV];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int64_t q = q0 + u;
                cidx[u] = 0;
                cval[u] = T(0);
                if (q < ce) {
                    cidx[u] = ld_stream(a.indices + q, ps);
                    cval[u] = ld_stream(a.data + q, ps);
                }
            }
#pragma unroll
            for (int u = 0; u < U; ++u)
#pragma unroll
                for (int m = 0; m < NCV; ++m) {
                    const int64_t col = ((int64_t)lane + (int64_t)m * G) * VEC;
#pragma unroll
                    for (int e = 0; e < VEC; ++e) b[u][m].v[e] = T(0);
                    if (q0 + u < ce && col < a.kt) b[u][m] = ld_gather_vec<T, VEC>(a.B + cidx[u] * a.ld + col, pg);
                }
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int64_t q = q0 + u;
                if (q < ce) {
                    if constexpr (MERGE) {
                        while (nxt <= q) {
                            if (first && head) {
                                store_row<T, G, VEC, NCV>(a.head + unit * a.kpart, acc, lane, a.kt);
                                split_arrive_rows<T, G, VEC, NCV>(a, r, a.indptr[r] / a.S, (nxt - 1) / a.S, lane,
                                                                  gmask);
                            } else if (r < a.row_limit) {
                                store_row<T, G, VEC, NCV>(a.C + r * a.ld, acc, lane, a.kt);
                            }
                            first = false;
                            acc.zero();
                            ++r;
                            nxt = a.indptr[r + 1];
                        }
                    }
#pragma unroll
                    for (int m = 0; m < NCV; ++m)
#pragma unroll
                        for (int e = 0; e < VEC; ++e) acc.v[m][e].mad(cval[u], b[u][m].v[e]);
                }
            }
        }
        if constexpr (MERGE) {
            if (nxt == ce) {
                if (first && head) {
                    store_row<T, G, VEC, NCV>(a.head + unit * a.kpart, acc, lane, a.kt);
                    split_arrive_rows<T, G, VEC, NCV>(a, r, a.indptr[r] / a.S, (nxt - 1) / a.S, lane, gmask);
                } else if (r < a.row_limit) {
                    store_row<T, G, VEC, NCV>(a.C + r * a.ld, acc, lane, a.kt);
                }
                if (ce == a.nnz) {
                    acc.zero();
                    for (int64_t rr = r + 1; rr < a.rows && rr < a.row_limit; ++rr)
                        store_row<T, G, VEC, NCV>(a.C + rr * a.ld, acc, lane, a.kt);
                }
            } else if (first && head) {
                store_row<T, G, VEC, NCV>(a.head + unit * a.kpart, acc, lane, a.kt);
                split_arrive_rows<T, G, VEC, NCV>(a, r, a.indptr[r] / a.S, (nxt - 1) / a.S, lane, gmask);
            } else {
                store_row<T, G, VEC, NCV>(a.tail + unit * a.kpart, acc, lane, a.kt);
                split_arrive_rows<T, G, VEC, NCV>(a, r, unit, (nxt - 1) / a.S, lane, gmask);
            }
        } else {
            if (r < a.row_limit) store_row<T, G, VEC, NCV>(a.C + r * a.ld, acc, lane, a.kt);
        }
    }
}

// ------------------------------------------------------------------ SDDMM
template <typename T, int G, int VEC, int NCV, int U, bool MERGE>
__global__ void __launch_bounds__(512) sddmm_kernel(DenseArgs<T> a) {
    const int lane = threadIdx.x % G;
    const unsigned gmask = group_mask<G>();
    const int64_t gid = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) / G;
    const int64_t ngroups = ((int64_t)gridDim.x * blockDim.x) / G;
    const uint64_t ps = policy_evict_first();
    const uint64_t pg = policy_evict_last();

    for (int64_t unit = gid; unit < a.nunits; unit += ngroups) {
        int64_t cs, ce, r, nxt;
        if constexpr (MERGE) {
            cs = unit * a.S;
            ce = min(cs + a.S, a.nnz);
            r = chunk_first_row(a.indptr, a.own_first, a.rows, unit, cs);
            nxt = a.indptr[r + 1];
        } else {
            r = unit;
            cs = a.indptr[r];
            ce = a.indptr[r + 1];
            nxt = ce;
        }
        for (int64_t q0 = cs; q0 < ce; q0 += U) {
            int64_t cidx[U], crow[U];
            T cval[U];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int64_t q = q0 + u;
                cidx[u] = 0;
                cval[u] = T(0);
                crow[u] = r;
                if (q < ce) {
                    cidx[u] = ld_stream(a.indices + q, ps);
                    if (a.pass == kPassOnly || a.pass == kPassLast) cval[u] = ld_stream(a.data + q, ps);
                    if constexpr (MERGE) {
                        while (nxt <= q) {
                            ++r;
                            nxt = a.indptr[r + 1];
                        }
                    }
                    crow[u] = r;
                }
            }
            Sum<T> dot[U];
            for (int64_t kb = 0; kb < a.kt; kb += (int64_t)G * VEC * NCV) {
#pragma unroll
            for (int u = 0; u < U; ++u) {
#pragma unroll
                for (int m = 0; m < NCV; ++m) {
                    const int64_t col = kb + ((int64_t)lane + (int64_t)m * G) * VEC;
                    if (q0 + u < ce && col < a.kt) {
                        const Vec<T, VEC> vv = ld_gather_vec<T, VEC>(a.B + cidx[u] * a.ld + col, pg);
                        const Vec<T, VEC> uu = ld_gather_vec<T, VEC>(a.U + crow[u] * a.ld + col, pg);
#pragma unroll
                        for (int e = 0; e < VEC; ++e) dot[u].mad(uu.v[e], vv.v[e]);
                    }
                }
            }
            }
#pragma unroll
            for (int u = 0; u < U; ++u) {
                T d = group_sum<G>(dot[u].get(), gmask);
                const int64_t q = q0 + u;
                if (lane == (u % G) && q < ce && crow[u] < a.row_limit) {
                    if (a.pass == kPassOnly) {
                        a.C[q] = cval[u] * d;
                    } else if (a.pass == kPassFirst) {
                        a.C[q] = d;
                    } else if (a.pass == kPassMid) {
                        a.C[q] += d;
                    } else {
                        a.C[q] = cval[u] * (a.C[q] + d);
                    }
                }
            }
        }
    }
}

}  // namespace tg
