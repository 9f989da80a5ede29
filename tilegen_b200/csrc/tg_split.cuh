// nnz-balanced chunking shared by the merge-split kernels (SpMV, SpMM, SDDMM).
//
// The nonzeros are cut into chunks of S consecutive positions: chunk c covers
// [c*S, min((c+1)*S, nnz)).  A row is OWNED by the chunk that holds its first
// position (empty rows: the chunk holding their start offset; rows whose start is nnz
// belong to the last chunk), so every output row has exactly one writer.
//
// own_first[c] = first row r with indptr[r] >= c*S (a lower bound into indptr), for
// c in [0, nchunks); own_first[nchunks] = rows.  It is produced by one streaming pass
// over indptr (partition_kernel), which is the only "analysis" the merge path needs.
//
// A row whose nonzeros cross chunk boundaries (a SPLIT row spanning chunks ca..cb) gets
// one partial sum per chunk: tail[ca] from its owner, head[c] from each later chunk, and
// the row is tail[ca] + head[ca+1] + ... + head[cb] in that fixed order (deterministic).
// The partials are summed in place: every contributor publishes its partial and arrives
// on one counter of the row (SpMV: cnt[cb], with an acq_rel atomic; SpMM/SDDMM: cnt[ca],
// after a fence), and the last of the (cb - ca + 1) arrivals adds them, writes the row
// and resets the counter to zero, so the counters are zero after every call.
#pragma once

#include "tg_common.cuh"

namespace tg {

// Workspace layout of the merge path; every sub-buffer is 256-byte aligned.
struct SplitWs {
    int64_t* own_first;  // [nchunks + 1]
    int* cnt;            // [nchunks]
    void* head;          // [nchunks * width] partials (value type of the op)
    void* tail;          // [nchunks * width]
    uint32_t* err;       // [1] device error word (bounded waits, bounds checks)
};

inline size_t align256(size_t b) { return (b + 255) & ~size_t(255); }

inline size_t split_ws_bytes(int64_t nchunks, int64_t width, size_t elem) {
    return align256(sizeof(int64_t) * (nchunks + 1)) + align256(sizeof(int) * (nchunks > 0 ? nchunks : 1)) +
           2 * align256(elem * (size_t)(nchunks > 0 ? nchunks : 1) * (size_t)width) + align256(sizeof(uint32_t));
}

inline SplitWs split_ws_carve(void* base, int64_t nchunks, int64_t width, size_t elem) {
    char* p = static_cast<char*>(base);
    SplitWs w;
    w.own_first = reinterpret_cast<int64_t*>(p);
    p += align256(sizeof(int64_t) * (nchunks + 1));
    w.cnt = reinterpret_cast<int*>(p);
    p += align256(sizeof(int) * (nchunks > 0 ? nchunks : 1));
    w.head = p;
    p += align256(elem * (size_t)(nchunks > 0 ? nchunks : 1) * (size_t)width);
    w.tail = p;
    p += align256(elem * (size_t)(nchunks > 0 ? nchunks : 1) * (size_t)width);
    w.err = reinterpret_cast<uint32_t*>(p);
    return w;
}

// One thread per row boundary r in [0, rows]: sets own_first[c] for every chunk c
// whose first position c*S lies in (indptr[r-1], indptr[r]]; zeroes the arrival
// counters and the error word.  It lets a kernel launched after it with programmatic
// serialisation start at once (that kernel waits with pdl_wait before reading the table).
__global__ void partition_kernel(const int64_t* __restrict__ indptr, int64_t rows, int64_t S, int64_t nchunks,
                                 int64_t* __restrict__ own_first, int* __restrict__ cnt, uint32_t* err);

// Host launcher (defined in tg_split.cu).
int launch_partition(const int64_t* indptr, int64_t rows, int64_t nnz, int64_t S, const SplitWs& ws,
                     cudaStream_t stream);

}  // namespace tg
