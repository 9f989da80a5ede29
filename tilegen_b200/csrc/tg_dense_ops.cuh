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
    const int64_t* own_first;
    int* cnt;
    T* head;
    T* tail;
};

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
                    cval[u] = ld_stream(a.data + q, ps);
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
                if (lane == (u % G) && q < ce && crow[u] < a.row_limit) a.C[q] = cval[u] * d;
            }
        }
    }
}

}  // namespace tg

namespace tg {

// ------------------------------------------------------------------ row groups
// Block-structured matrices (the reference corpus's `blocked` class, dense 8x8 blocks,
// tilegen/matrices.py:135-161; BSR in tilegen/ir.py:101) store, in CSR, runs of
// consecutive rows with identical column lists.  With TG_SPLIT_BLOCK the SpMM works on
// GROUPS of kGroupRows consecutive rows: a plan pass flags every group whose rows share
// one column list, and for a flagged group one warp gathers each dense row B[j, :] ONCE
// and applies it to all of the group's rows (kGroupRows x fewer gathers); other groups
// are done row by row by the same warp.  Each row is summed over its nonzeros in index
// order, as in the rowwise kernel, so the results are the same.
constexpr int kGroupRows = 8;

// flag[g] = 1 when rows [g*R, g*R + R) all exist and have the same column list.  One
// warp per group; lanes stride over the positions.
template <int R>
__global__ void __launch_bounds__(256) group_plan_kernel(const int64_t* __restrict__ indptr,
                                                         const int64_t* __restrict__ indices, int64_t rows,
                                                         int64_t ngroups, uint8_t* __restrict__ flag) {
    const int lane = threadIdx.x % kWarp;
    const int64_t nw = ((int64_t)gridDim.x * blockDim.x) / kWarp;
    for (int64_t g = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) / kWarp; g < ngroups; g += nw) {
        const int64_t r0 = g * R;
        bool same = r0 + R <= rows;
        if (same) {
            const int64_t p0 = indptr[r0];
            const int64_t len = indptr[r0 + 1] - p0;
            for (int r = 1; r < R && same; ++r) {
                const int64_t pr = indptr[r0 + r];
                if (indptr[r0 + r + 1] - pr != len) {
                    same = false;
                    break;
                }
                bool ok = true;
                for (int64_t q = lane; q < len; q += kWarp) ok &= (indices[p0 + q] == indices[pr + q]);
                same = __all_sync(kFull, ok);
            }
        }
        if (lane == 0) flag[g] = same ? 1 : 0;
    }
}

// One warp per (group, column slice) task, grid-stride; the slices of a group go to
// neighbouring warps, which share the group's index and value loads through L1.  Lane l
// owns the VEC columns s + l*VEC of slice s (32*VEC columns).  Positions are read 32 at a
// time (one coalesced load of indices and of each row's values per 32 positions) and
// handed out by shuffles; UG gathers are in flight per lane.
template <typename T, int VEC, int UG>
__global__ void __launch_bounds__(256) spmm_group_kernel(DenseArgs<T> a, const uint8_t* __restrict__ flag,
                                                         int64_t ngroups) {
    constexpr int R = kGroupRows;
    const int lane = threadIdx.x % kWarp;
    const int64_t nw = ((int64_t)gridDim.x * blockDim.x) / kWarp;
    const uint64_t ps = policy_evict_first();
    const uint64_t pg = policy_evict_last();
    const int64_t nslices = (a.kt + (int64_t)kWarp * VEC - 1) / ((int64_t)kWarp * VEC);
    for (int64_t task = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) / kWarp; task < ngroups * nslices;
         task += nw) {
        const int64_t g = task / nslices;
        const int64_t r0 = g * R;
        const bool grouped = flag[g] != 0;
        const int nrows = (int)min((int64_t)R, a.rows - r0);
        {
            const int64_t s0 = (task % nslices) * (int64_t)kWarp * VEC;
            const int64_t col = s0 + (int64_t)lane * VEC;
            const bool live = col < a.kt;
            if (grouped) {
                // the rows of a flagged group have one column list, hence one length:
                // row r starts at base + r * len
                const int64_t base = a.indptr[r0];
                const int64_t len = a.indptr[r0 + 1] - base;
                Sum<T> acc[R][VEC];
                for (int64_t p0 = 0; p0 < len; p0 += kWarp) {
                    const int n = (int)min((int64_t)kWarp, len - p0);
                    int64_t myidx = 0;
                    T myval[R];
                    if (lane < n) myidx = ld_stream(a.indices + base + p0 + lane, ps);
#pragma unroll
                    for (int r = 0; r < R; ++r)
                        myval[r] = lane < n ? ld_stream(a.data + base + r * len + p0 + lane, ps) : T(0);
                    for (int j0 = 0; j0 < n; j0 += UG) {
                        Vec<T, VEC> b[UG];
#pragma unroll
                        for (int u = 0; u < UG; ++u) {
                            const int64_t c = __shfl_sync(kFull, myidx, (j0 + u) & 31);
#pragma unroll
                            for (int e = 0; e < VEC; ++e) b[u].v[e] = T(0);
                            if (live && j0 + u < n) b[u] = ld_gather_vec<T, VEC>(a.B + c * a.ld + col, pg);
                        }
#pragma unroll
                        for (int u = 0; u < UG; ++u) {
                            if (j0 + u < n) {  // warp-uniform
#pragma unroll
                                for (int r = 0; r < R; ++r) {
                                    const T v = __shfl_sync(kFull, myval[r], j0 + u);
#pragma unroll
                                    for (int e = 0; e < VEC; ++e) acc[r][e].mad(v, b[u].v[e]);
                                }
                            }
                        }
                    }
                }
                if (live) {
#pragma unroll
                    for (int r = 0; r < R; ++r) {
                        if (r0 + r < a.row_limit) {
                            Vec<T, VEC> o;
#pragma unroll
                            for (int e = 0; e < VEC; ++e) o.v[e] = acc[r][e].get();
                            st_vec<T, VEC>(a.C + (r0 + r) * a.ld + col, o);
                        }
                    }
                }
            } else {
                for (int r = 0; r < nrows; ++r) {
                    const int64_t rr = r0 + r;
                    const int64_t pb = a.indptr[rr], pe = a.indptr[rr + 1];
                    Sum<T> acc[VEC];
                    for (int64_t p0 = pb; p0 < pe; p0 += kWarp) {
                        const int n = (int)min((int64_t)kWarp, pe - p0);
                        int64_t myidx = 0;
                        T myval = T(0);
                        if (lane < n) {
                            myidx = ld_stream(a.indices + p0 + lane, ps);
                            myval = ld_stream(a.data + p0 + lane, ps);
                        }
                        for (int j0 = 0; j0 < n; j0 += UG) {
                            Vec<T, VEC> b[UG];
#pragma unroll
                            for (int u = 0; u < UG; ++u) {
                                const int64_t c = __shfl_sync(kFull, myidx, (j0 + u) & 31);
#pragma unroll
                                for (int e = 0; e < VEC; ++e) b[u].v[e] = T(0);
                                if (live && j0 + u < n) b[u] = ld_gather_vec<T, VEC>(a.B + c * a.ld + col, pg);
                            }
#pragma unroll
                            for (int u = 0; u < UG; ++u) {
                                if (j0 + u < n) {
                                    const T v = __shfl_sync(kFull, myval, j0 + u);
#pragma unroll
                                    for (int e = 0; e < VEC; ++e) acc[e].mad(v, b[u].v[e]);
                                }
                            }
                        }
                    }
                    if (live && rr < a.row_limit) {
                        Vec<T, VEC> o;
#pragma unroll
                        for (int e = 0; e < VEC; ++e) o.v[e] = acc[e].get();
                        st_vec<T, VEC>(a.C + rr * a.ld + col, o);
                    }
                }
            }
        }
    }
}

}  // namespace tg
