// Host-side parameter selection and template dispatch for SpMM / SDDMM.
//
// Knob mapping (the reference's SpMM/SDDMM emitters only consume T, so the b200 meaning
// of the other knobs is defined here):
//   TPR -> G, lanes per group (clamped to 4..32 and to the lanes the row width can use),
//   V   -> VEC, elements per gather (largest of {4,2,1} <= V that divides K and the
//          operand alignment; 2 at most for fp64),
//   U   -> nonzeros whose gathers are in flight per group (1, 2 or 4),
//   B   -> threads per CTA (128, 256 or 512),
//   split / chunk_nnz -> rowwise (one group per row) or merge (one group per chunk);
//          block (SpMM): a warp per group of kGroupRows rows sharing each gathered row;
//          SDDMM takes block as merge.
#pragma once

#include <algorithm>

#include "tg_dense_ops.cuh"

namespace tg {

struct DenseChoice {
    int G, VEC, NCV, U, block;
    bool merge;
    int64_t S;
    int64_t ktile;  // SpMM columns per launch (what a lane group's accumulators cover)
};

inline int pow2_floor(int v) {
    int p = 1;
    while (p * 2 <= v) p *= 2;
    return p;
}
inline int pow2_ceil(int64_t v) {
    int p = 1;
    while (p < v) p *= 2;
    return p;
}

inline bool aligned_to(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// Default merge chunk.  SpMM: 256 nonzeros per lane group, since each chunk boundary
// inside a row costs a K-wide partial and its fix-up (on C5, 64 / 128 / 256 / 384
// nonzeros: 2.09 / 1.84 / 1.75 / 1.74 ms).  SDDMM has no row sums to split, so small
// chunks cost it nothing and give more lane groups, each with its own chain of row
// gathers in flight: 64 nonzeros, halved (down to 32) until the call has at least 32768
// chunks, so that a small matrix (or one GPU's shard of a large one) still fills every SM
// (C5 SDDMM, 32 / 64 / 128 / 256 nonzeros: 1.05-1.10 / 1.06 / 1.15 / 1.32 ms).  A function
// of nnz and the op alone, so that the workspace size and the launch agree.
inline int64_t default_dense_chunk(int64_t nnz, bool is_spmm) {
    if (is_spmm) return 256;
    int64_t S = 64;
    while (S > 32 && nnz / S < 32768) S /= 2;
    return S;
}

template <typename T>
DenseChoice choose_dense(const tg_sched& s, int64_t K, bool is_spmm, const void* p0, const void* p1, int64_t nnz) {
    DenseChoice d{};
    const int vmax = sizeof(T) == 4 ? 4 : 2;
    int vec = std::min(std::max(s.vector_width, 1), vmax);
    vec = pow2_floor(vec);
    while (vec > 1 && (K % vec != 0 || !aligned_to(p0, vec * sizeof(T)) || !aligned_to(p1, vec * sizeof(T))))
        vec /= 2;
    d.VEC = vec;
    const int64_t nvec = (K + vec - 1) / vec;  // column vectors per row
    int g = pow2_floor(std::min(std::max(s.threads_per_row, 4), 32));
    g = std::max(4, std::min(g, pow2_ceil(nvec)));
    d.G = g;
    const int64_t per_lane = (nvec + g - 1) / g;
    d.NCV = per_lane <= 1 ? 1 : (per_lane <= 2 ? 2 : 4);
    // SpMM covers at most G*VEC*NCV columns per launch (its accumulators live in
    // registers); SDDMM loops over all K columns inside the kernel
    d.ktile = is_spmm ? std::min<int64_t>(K, (int64_t)g * vec * d.NCV) : K;
    d.U = s.unroll >= 4 ? 4 : (s.unroll >= 2 ? 2 : 1);
    d.block = (s.block_size >= 512) ? 512 : (s.block_size >= 256 ? 256 : 128);
    d.merge = (s.split == TG_SPLIT_MERGE || s.split == TG_SPLIT_STREAM || s.split == TG_SPLIT_BLOCK);
    d.S = s.chunk_nnz > 0 ? s.chunk_nnz : default_dense_chunk(nnz, is_spmm);
    return d;
}

template <typename T, int G, int VEC, int NCV, int U, bool MERGE>
void launch_dense(bool is_spmm, const DenseArgs<T>& a, int block, cudaStream_t st) {
    int64_t groups_per_block = block / G;
    int64_t blocks = ceil_div(a.nunits, groups_per_block);
    if (blocks > 148 * 64) blocks = 148 * 64;
    if (blocks < 1) blocks = 1;
    if (is_spmm)
        spmm_kernel<T, G, VEC, NCV, U, MERGE><<<(unsigned)blocks, block, 0, st>>>(a);
    else
        sddmm_kernel<T, G, VEC, NCV, U, MERGE><<<(unsigned)blocks, block, 0, st>>>(a);
}

template <typename T, int G, int VEC, int NCV, int U>
bool dense_m(const DenseChoice& d, bool sp, const DenseArgs<T>& a, cudaStream_t st) {
    if (d.merge)
        launch_dense<T, G, VEC, NCV, U, true>(sp, a, d.block, st);
    else
        launch_dense<T, G, VEC, NCV, U, false>(sp, a, d.block, st);
    return true;
}

template <typename T, int G, int VEC, int NCV>
bool dense_u(const DenseChoice& d, bool sp, const DenseArgs<T>& a, cudaStream_t st) {
    switch (d.U) {
        case 1: return dense_m<T, G, VEC, NCV, 1>(d, sp, a, st);
        case 2: return dense_m<T, G, VEC, NCV, 2>(d, sp, a, st);
        case 4: return dense_m<T, G, VEC, NCV, 4>(d, sp, a, st);
    }
    return false;
}

template <typename T, int G, int VEC>
bool dense_n(const DenseChoice& d, bool sp, const DenseArgs<T>& a, cudaStream_t st) {
    switch (d.NCV) {
        case 1: return dense_u<T, G, VEC, 1>(d, sp, a, st);
        case 2: return dense_u<T, G, VEC, 2>(d, sp, a, st);
        case 4: return dense_u<T, G, VEC, 4>(d, sp, a, st);
    }
    return false;
}

template <typename T, int G>
bool dense_v(const DenseChoice& d, bool sp, const DenseArgs<T>& a, cudaStream_t st) {
    switch (d.VEC) {
        case 1: return dense_n<T, G, 1>(d, sp, a, st);
        case 2: return dense_n<T, G, 2>(d, sp, a, st);
        case 4:
            if constexpr (sizeof(T) == 4) return dense_n<T, G, 4>(d, sp, a, st);
            return false;
    }
    return false;
}

template <typename T>
bool dense_dispatch(const DenseChoice& d, bool sp, const DenseArgs<T>& a, cudaStream_t st) {
    switch (d.G) {
        case 4: return dense_v<T, 4>(d, sp, a, st);
        case 8: return dense_v<T, 8>(d, sp, a, st);
        case 16: return dense_v<T, 16>(d, sp, a, st);
        case 32: return dense_v<T, 32>(d, sp, a, st);
    }
    return false;
}

// SpMM with TG_SPLIT_BLOCK: the group plan (one flag byte per group of kGroupRows rows).
inline bool block_split(const tg_sched& s, bool is_spmm) { return is_spmm && s.split == TG_SPLIT_BLOCK; }

template <typename T>
size_t dense_ws_bytes(int64_t rows, int64_t nnz, int64_t K, const tg_sched& s, bool is_spmm) {
    if (block_split(s, is_spmm)) return rows > 0 ? align256((size_t)ceil_div(rows, kGroupRows)) : 0;
    if ((s.split != TG_SPLIT_MERGE && s.split != TG_SPLIT_STREAM && s.split != TG_SPLIT_BLOCK) || nnz <= 0 || K <= 0)
        return 0;
    // alignment does not change the partial width's upper bound: size for the widest tile
    const DenseChoice d = choose_dense<T>(s, K, is_spmm, nullptr, nullptr, nnz);
    const int64_t nchunks = ceil_div(nnz, d.S);
    const int64_t width = is_spmm ? (int64_t)d.G * (sizeof(T) == 4 ? 4 : 2) * 4 : 0;
    return split_ws_bytes(nchunks, width, sizeof(T));
}

// SpMM: one launch per slab of G*VEC*NCV columns (the accumulators of a lane group
// cover that many); SDDMM: one launch.
template <typename T>
int launch_tiles(const DenseChoice& d, bool is_spmm, const DenseArgs<T>& a, const T* B, const T* U, T* C, int64_t K,
                 cudaStream_t st) {
    for (int64_t k0 = 0; k0 < (is_spmm ? K : 1); k0 += d.ktile) {
        DenseArgs<T> t = a;
        t.B = B + (is_spmm ? k0 : 0);
        t.U = U;
        t.C = C + (is_spmm ? k0 : 0);
        t.kt = is_spmm ? std::min(d.ktile, K - k0) : K;
        if (!dense_dispatch<T>(d, is_spmm, t, st))
            return set_error(TG_EUNSUPPORTED, "no %s instance for G=%d VEC=%d NCV=%d U=%d", is_spmm ? "spmm" : "sddmm",
                             d.G, d.VEC, d.NCV, d.U);
        int rc = check_launch(is_spmm ? "spmm_kernel" : "sddmm_kernel");
        if (rc != TG_OK) return rc;
    }
    return TG_OK;
}

// SpMM over row groups (TG_SPLIT_BLOCK): plan unless reused, then one launch (the
// warps loop over K in slices of 32*VEC columns).
template <typename T>
int spmm_groups_run(const tg_csr& A, const T* B, T* C, int64_t K, const tg_sched& s, void* ws, size_t ws_bytes,
                    cudaStream_t st) {
    const int64_t ngroups = ceil_div(A.rows, kGroupRows);
    const size_t need = align256((size_t)ngroups);
    if (ws == nullptr || ws_bytes < need)
        return set_error(TG_ENOMEM, "spmm block split needs %zu workspace bytes, got %zu", need, ws_bytes);
    uint8_t* flag = static_cast<uint8_t*>(ws);
    const int64_t warps_per_cta = 256 / kWarp;
    const int64_t blocks = std::max<int64_t>(1, std::min<int64_t>(ceil_div(ngroups, warps_per_cta), 148 * 32));
    if (!(s.flags & TG_FLAG_REUSE_PLAN)) {
        group_plan_kernel<kGroupRows><<<(unsigned)blocks, 256, 0, st>>>(A.indptr, A.indices, A.rows, ngroups, flag);
        const int rc = check_launch("group_plan_kernel");
        if (rc != TG_OK) return rc;
    }
    // one 16-byte vector per lane (128 fp32 / 64 fp64 columns per warp task): splitting a
    // group's columns over more warps repeats its index and value loads and shuffles per
    // warp, which measured slower on the blocked class (73.2 vs 67.6 us)
    int vec = sizeof(T) == 4 ? 4 : 2;
    while (vec > 1 && (K % vec != 0 || !aligned_to(B, vec * sizeof(T)) || !aligned_to(C, vec * sizeof(T)))) vec /= 2;
    const int64_t tasks = ngroups * ceil_div(K, (int64_t)vec * kWarp);
    const int64_t blocks_run = std::max<int64_t>(1, std::min<int64_t>(ceil_div(tasks, warps_per_cta), 148 * 32));
    DenseArgs<T> a{};
    a.indptr = A.indptr;
    a.indices = A.indices;
    a.data = static_cast<const T*>(A.data);
    a.rows = A.rows;
    a.nnz = A.nnz;
    a.ld = K;
    a.row_limit = (s.flags & TG_FLAG_INJECT_BUG) ? A.rows - 1 : A.rows;
    a.B = B;
    a.C = C;
    a.kt = K;
    if (vec == 4) {
        if constexpr (sizeof(T) == 4) spmm_group_kernel<T, 4, 4><<<(unsigned)blocks_run, 256, 0, st>>>(a, flag, ngroups);
    } else if (vec == 2) {
        spmm_group_kernel<T, 2, 4><<<(unsigned)blocks_run, 256, 0, st>>>(a, flag, ngroups);
    } else {
        spmm_group_kernel<T, 1, 4><<<(unsigned)blocks_run, 256, 0, st>>>(a, flag, ngroups);
    }
    return check_launch("spmm_group_kernel");
}

// C = A * B (SpMM) or out = A .* (U V^T) on A's pattern (SDDMM, B = V).
template <typename T>
int dense_run(bool is_spmm, const tg_csr& A, const T* B, const T* U, T* C, int64_t K, const tg_sched& s, void* ws,
              size_t ws_bytes, cudaStream_t st) {
    if (K <= 0) return set_error(TG_EINVAL, "dense width K must be positive (got %lld)", (long long)K);
    if (A.rows == 0) return TG_OK;
    if (block_split(s, is_spmm)) return spmm_groups_run<T>(A, B, C, K, s, ws, ws_bytes, st);
    const DenseChoice d = choose_dense<T>(s, K, is_spmm, B, is_spmm ? (const void*)C : (const void*)U, A.nnz);
    DenseArgs<T> a{};
    a.indptr = A.indptr;
    a.indices = A.indices;
    a.data = static_cast<const T*>(A.data);
    a.rows = A.rows;
    a.nnz = A.nnz;
    a.ld = K;
    a.row_limit = (s.flags & TG_FLAG_INJECT_BUG) ? A.rows - 1 : A.rows;
    a.S = d.S;
    if (!is_spmm && A.nnz == 0) return TG_OK;
    if (d.merge && A.nnz > 0) {
        const int64_t nchunks = ceil_div(A.nnz, d.S);
        const int64_t width = is_spmm ? (int64_t)d.G * (sizeof(T) == 4 ? 4 : 2) * 4 : 0;
        const size_t need = split_ws_bytes(nchunks, width, sizeof(T));
        if (ws == nullptr || ws_bytes < need)
            return set_error(TG_ENOMEM, "%s merge split needs %zu workspace bytes, got %zu", is_spmm ? "spmm" : "sddmm",
                             need, ws_bytes);
        SplitWs w = split_ws_carve(ws, nchunks, width, sizeof(T));
        int rc = launch_partition(A.indptr, A.rows, A.nnz, d.S, w, st);
        if (rc != TG_OK) return rc;
        a.own_first = w.own_first;
        a.cnt = w.cnt;
        a.head = static_cast<T*>(w.head);
        a.tail = static_cast<T*>(w.tail);
        a.nunits = nchunks;
        a.kpart = (int64_t)d.G * d.VEC * d.NCV;
    } else {
        DenseChoice dr = d;
        dr.merge = false;
        a.nunits = A.rows;
        a.kpart = (int64_t)d.G * d.VEC * d.NCV;
        if (is_spmm && A.nnz == 0) {
            // every row is empty: C = 0 through the rowwise kernel (it writes empty rows)
        }
        return launch_tiles<T>(dr, is_spmm, a, B, U, C, K, st);
    }
    return launch_tiles<T>(d, is_spmm, a, B, U, C, K, st);
}

}  // namespace tg
