/*
 * tilegen_b200.h -- C ABI of libtilegen_b200.so, the sm_100a (B200) sparse hot path.
 *
 * Two layers are exported:
 *
 *  1. Reference-compatible launchers.  `launch_spmv`, `launch_spmm`, `launch_sddmm`,
 *     `launch_fused_spmv_axpy` and `launch_axpy` have exactly the signatures that
 *     TileGen's code generator emits (tilegen/codegen.py:226-280, ctypes argtypes in
 *     tilegen/verify.py:166-173).  Like the reference they take DEVICE pointers owned
 *     by the caller (tilegen/verify.py:414-420), run on the legacy default stream and
 *     end with a device-wide synchronize (tilegen/codegen.py:798), so
 *     `tilegen.verify.run_kernel` and `tilegen.autotune._make_caller` can drive them
 *     unchanged.  They read the schedule set by `tg_set_schedule` (process-global).
 *     Differences from the reference, all in the safe direction: SpMM writes C
 *     instead of accumulating into it (a caller that pre-zeroes C, as
 *     tilegen/verify.py:437 does, sees the same result), and the status of the last
 *     call is kept for `tg_last_status` / `tg_last_error_string`.
 *
 *  2. The native API (`tg_*`).  Asynchronous on the given CUDA stream, no internal
 *     synchronisation, no allocation: the caller passes a workspace of
 *     `tg_*_workspace_bytes(...)` bytes (NULL/0 when that size is 0).  Every call
 *     returns TG_OK (0) or a negative TG_E* status; the message is available from
 *     `tg_last_error_string()` on the calling host thread.  Calls on distinct
 *     streams/devices from distinct host threads are safe.
 *
 * Layout of the sparse operand (identical to the reference, tilegen/verify.py:318-335):
 * CSR with int64 `indptr[rows+1]` (non-decreasing, indptr[0] == 0, indptr[rows] == nnz),
 * int64 `indices[nnz]` in [0, cols) and values `data[nnz]`.  Dense operands are
 * row-major and contiguous.  All pointers are device pointers.
 */
#ifndef TILEGEN_B200_H
#define TILEGEN_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define TG_API __attribute__((visibility("default")))
#else
#define TG_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---------------------------------------------------------------- status codes */
#define TG_OK 0
#define TG_EINVAL -1       /* bad argument (null pointer, negative size, bad schedule) */
#define TG_ECUDA -2        /* a CUDA runtime call or kernel launch failed */
#define TG_ENOMEM -3       /* workspace too small, or the library's own allocation failed */
#define TG_EUNSUPPORTED -4 /* no kernel instance for this schedule / device */
#define TG_ETIMEDOUT -5    /* a bounded device-side wait ran out (multi-GPU paths) */
#define TG_EBOUNDS -6      /* bounds checking found an index out of range */

/* CUDA stream handle (a cudaStream_t); NULL is the legacy default stream. */
typedef void* tg_stream_t;

/* ------------------------------------------------------------------ schedule */
/* Row-to-thread mapping of the kernels. */
#define TG_SPLIT_ROWWISE 0 /* reference mapping: T rows per CTA tile, TPR lanes per row */
#define TG_SPLIT_MERGE 1   /* nnz-balanced chunks; a row split across chunks is finished by
                              its last contributor */
#define TG_SPLIT_AUTO 2    /* library picks: the merge split (any row-length distribution) */
#define TG_SPLIT_STREAM 3  /* SpMV: persistent TMA-fed row-block kernel; merge for SpMM/SDDMM */
#define TG_SPLIT_BLOCK 4   /* SpMM: groups of 8 consecutive rows with one shared column list
                              (block-structured matrices) gather each dense row once for the
                              whole group; other groups row by row.  Merge for SpMV/SDDMM. */

/* flags */
#define TG_FLAG_BOUNDS_CHECK 1u /* validate indptr/indices on the device; TG_EBOUNDS on error */
#define TG_FLAG_INJECT_BUG 2u   /* deliberately skip the last row (harness self-test) */
#define TG_FLAG_INDEX32 8u      /* power steps (tg_power_step_f64, tg_power_step_p2p_f64):
                                   A.indices points to int32 column indices (renumbered by
                                   tg_renumber_columns_i32); rowwise split, no bounds check */
#define TG_FLAG_REUSE_PLAN 4u   /* SpMV merge / stream and SpMM block splits: the workspace
                                   already holds this matrix's plan (partition or row-group
                                   flags) from an earlier call with the same A and schedule;
                                   skip the analysis pass */

/*
 * Mirrors tilegen.codegen.Lowering (tilegen/codegen.py:90-134): each knob of the
 * reference's Config/schedule IR is one field here and one template parameter of
 * the kernels.  Zero in any field selects the library default for that knob.
 */
typedef struct tg_sched {
    int32_t tile;            /* T: rows per CTA tile (Tile, passes.py:243-270)            */
    int32_t threads_per_row; /* TPR: lanes cooperating on one row (ThreadsPerRow)        */
    int32_t unroll;          /* U: independent loads in flight per lane (Unroll)          */
    int32_t vector_width;    /* V: elements per vector load (Vectorize)                   */
    int32_t block_size;      /* B: threads per CTA (Parallelize block_size), 32..512      */
    int32_t split;           /* TG_SPLIT_*                                                */
    int32_t chunk_nnz;       /* merge split: nonzeros per chunk (0 = library default)     */
    uint32_t flags;          /* TG_FLAG_*                                                 */
} tg_sched;

/* CSR operand; `data` is double* for *_f64 entry points and float* for *_f32. */
typedef struct tg_csr {
    int64_t rows;
    int64_t cols;
    int64_t nnz;
    const int64_t* indptr;
    const int64_t* indices;
    const void* data;
} tg_csr;

/* ------------------------------------------------------------ library / errors */
TG_API const char* tg_version(void);
/* Message for the last failing tg_* / launch_* call on this host thread ("" if none). */
TG_API const char* tg_last_error_string(void);
/* Status of the last reference-compatible launch_* call on this host thread. */
TG_API int tg_last_status(void);
/* Number of kernels this library has launched in the process so far (all threads and
 * devices; memsets and copies are not kernels).  Benchmarks difference it around a
 * timed region. */
TG_API uint64_t tg_launch_count(void);
/* Fills *s with the library defaults (reference BASELINE T32/TPR1/U1/V1/B128,
 * tilegen/autotune.py:55-56, with split = TG_SPLIT_ROWWISE). */
TG_API void tg_default_schedule(tg_sched* s);
/* Checks a schedule; returns TG_OK or TG_EINVAL (reason in tg_last_error_string). */
TG_API int tg_validate_schedule(const tg_sched* s);

/* Process-global schedule read by the launch_* shims (not by the tg_* API). */
TG_API int tg_set_schedule(const tg_sched* s);
TG_API int tg_get_schedule(tg_sched* s);

/* ----------------------------------------------------------- workspace sizing */
/* Bytes of device workspace needed by the tg_* call with the same arguments.
 * `k` is the dense width (K) for SpMM/SDDMM and 1 for SpMV. */
TG_API size_t tg_spmv_workspace_bytes(int64_t rows, int64_t nnz, const tg_sched* s);
TG_API size_t tg_spmm_workspace_bytes(int64_t rows, int64_t nnz, int64_t k, const tg_sched* s);
TG_API size_t tg_sddmm_workspace_bytes(int64_t rows, int64_t nnz, int64_t k, const tg_sched* s);

/* ------------------------------------------------------------------ native API */
/* y[i] = sum_p data[p] * x[indices[p]]          (ref: tilegen/codegen.py:592-643,
 * math cpp/src/ref.cpp:6-15). fp64 in, fp64 accumulate. */
TG_API int tg_spmv_f64(const tg_csr* A, const double* x, double* y, const tg_sched* s,
                void* workspace, size_t workspace_bytes, tg_stream_t stream);
/* fp32 values/x/y with fp32 accumulation (north_star: rel. error <= 1e-4). */
TG_API int tg_spmv_f32(const tg_csr* A, const float* x, float* y, const tg_sched* s,
                void* workspace, size_t workspace_bytes, tg_stream_t stream);
/* z[i] = alpha * (A x)[i] + beta * w[i]       (ref: tilegen/dsl.py:237-247 after
 * loop_fusion, tilegen/passes.py:188-240; math cpp/src/ref.cpp:62-73). */
TG_API int tg_fused_spmv_axpy_f64(const tg_csr* A, const double* x, const double* w, double* z,
                           double alpha, double beta, const tg_sched* s, void* workspace,
                           size_t workspace_bytes, tg_stream_t stream);
/* The same with fp32 values, x, w, z and fp32 accumulation (the reference DSL's dtype
 * "f32", tilegen/dsl.py:124-147; north_star: rel. error <= 1e-4). */
TG_API int tg_fused_spmv_axpy_f32(const tg_csr* A, const float* x, const float* w, float* z, float alpha,
                                  float beta, const tg_sched* s, void* workspace, size_t workspace_bytes,
                                  tg_stream_t stream);
/* C[i,:] = sum_p data[p] * B[indices[p],:]; B is cols x k, C is rows x k, row-major.
 * C is overwritten (ref: tilegen/codegen.py:646-685, math cpp/src/ref.cpp:31-43). */
TG_API int tg_spmm_f32(const tg_csr* A, const float* B, float* C, int64_t k, const tg_sched* s,
                void* workspace, size_t workspace_bytes, tg_stream_t stream);
TG_API int tg_spmm_f64(const tg_csr* A, const double* B, double* C, int64_t k, const tg_sched* s,
                void* workspace, size_t workspace_bytes, tg_stream_t stream);
/* out[p] = data[p] * dot(U[i,:], V[indices[p],:]) for p in row i; U is rows x k,
 * V is cols x k.  The output pattern is A's (indptr/indices unchanged)
 * (ref: tilegen/codegen.py:688-714, math cpp/src/ref.cpp:46-59). */
TG_API int tg_sddmm_f32(const tg_csr* A, const float* U, const float* V, float* out, int64_t k,
                 const tg_sched* s, void* workspace, size_t workspace_bytes,
                 tg_stream_t stream);
TG_API int tg_sddmm_f64(const tg_csr* A, const double* U, const double* V, double* out, int64_t k,
                 const tg_sched* s, void* workspace, size_t workspace_bytes,
                 tg_stream_t stream);
/* z = alpha * x + beta * w (ref: tilegen/dsl.py:250-256, tilegen/codegen.py:580-589). */
TG_API int tg_axpy_f64(const double* x, const double* w, double* z, double alpha, double beta,
                int64_t n, const tg_sched* s, tg_stream_t stream);
TG_API int tg_axpy_f32(const float* x, const float* w, float* z, float alpha, float beta, int64_t n,
                       const tg_sched* s, tg_stream_t stream);

/* ------------------------------------------------------ power iteration (new) */
/* Iterated SpMV x <- A x / ||A x||, one process per GPU, rows split into `nparts`
 * contiguous shards.  No counterpart in the reference (north_star's multi-GPU mode).
 * The iterate is a padded vector of nparts * stride doubles: shard r occupies
 * [r*stride, r*stride + rows_r) and its last element r*stride + stride - 1 (the slot)
 * holds sum(shard^2).  A's column indices must be renumbered to this layout
 * (j -> owner(j) * stride + j - first_row(owner)).  The workspace must be zero-filled
 * before its first use; every call leaves it zeroed. */
TG_API size_t tg_power_workspace_bytes(int64_t nnz, const tg_sched* s);
/* out[i] = owner(j) * stride + (j - bounds[owner(j)]) for j = indices[i], i < nnz: the
 * column renumbering above, on the device.  `bounds` (host memory, nparts + 1 <= 65
 * entries) are the row bounds of the shards, bounds[0] = 0, each shard shorter than
 * `stride`; the indices must lie in [0, bounds[nparts]).  out may equal indices. */
TG_API int tg_renumber_columns(const int64_t* indices, int64_t* out, int64_t nnz, const int64_t* bounds,
                               int32_t nparts, int64_t stride, tg_stream_t stream);
/* The same renumbering written as int32 (the padded layout nparts * stride must be below
 * 2^31): the power steps read it with TG_FLAG_INDEX32, 12 bytes of CSR stream per nonzero
 * instead of 16. */
TG_API int tg_renumber_columns_i32(const int64_t* indices, int32_t* out, int64_t nnz, const int64_t* bounds,
                                   int32_t nparts, int64_t stride, tg_stream_t stream);
/* y[0..rows) = A x / sqrt(sum of the nparts slots of x); y[stride-1] = sum(y^2). */
TG_API int tg_power_step_f64(const tg_csr* A, const double* x, int32_t nparts, int64_t stride,
                             double* y, const tg_sched* s, void* workspace,
                             size_t workspace_bytes, tg_stream_t stream);
/* shard[stride-1] = sum(shard[0..rows)^2) (slot of an initial iterate). */
TG_API int tg_shard_norm2_f64(double* shard, int64_t rows, int64_t stride, void* workspace,
                              size_t workspace_bytes, tg_stream_t stream);
/* x_out[0..rows) = shard `part` of x divided by sqrt(sum of slots); *lambda = that norm. */
TG_API int tg_power_finalize_f64(const double* x, int32_t nparts, int64_t stride, int32_t part,
                                 int64_t rows, double* x_out, double* lambda_out,
                                 tg_stream_t stream);

/* Power step fused with the shard exchange over peer memory (1..8 GPUs of one node).
 * y_peers[q] is rank q's next-iterate buffer (nparts * stride doubles) and flag_peers[q]
 * rank q's flag array (nparts uint64, zero-filled before the first epoch), both mapped
 * into this process (CUDA IPC); index `rank` is this rank's own.  The kernel waits
 * (bounded, 2 s) until flag_peers[rank][q] >= epoch-1 for every q, computes its shard
 * tile by tile and stores each tile into every y_peers[q], writes its slot to all
 * ranks, then stores `epoch` into flag_peers[q][rank] (system-scope release).  Call with
 * epoch = 1, 2, ... and alternate two iterate buffers.  A wait that runs out sets bit 4
 * (value 16) of the workspace's error word (read it with tg_power_error).  The error word
 * is sticky: while it is set, every step and tg_p2p_wait on this workspace returns at once
 * without computing, writing the slot or releasing a flag (so the peers give up in turn),
 * and the kernel always leaves the workspace's ticket at zero.  To restart, every rank
 * zeroes its flag array and calls tg_power_clear_error, then steps again from epoch 1.
 * Plain peer stores only: no multicast, no TMA. */
TG_API int tg_power_step_p2p_f64(const tg_csr* A, const double* x, int32_t nparts, int32_t rank,
                                 int64_t stride, double* const* y_peers, uint64_t* const* flag_peers,
                                 uint64_t epoch, const tg_sched* s, void* workspace,
                                 size_t workspace_bytes, tg_stream_t stream);
/* The power step with the exchange done by copy engines (the alternative to
 * tg_power_step_p2p_f64; same peer buffers, flags and epochs): wait (bounded, 2 s) until
 * every rank released epoch - 1; compute this rank's rows in `nchunks` (1..16) row chunks
 * into its own next-iterate buffer y_peers[rank], copying each chunk into every other
 * rank's buffer as soon as it is done (one copy per peer, on side streams the library keeps
 * per device, so the copies overlap the next chunk's compute); the slot (the chunks' sums
 * of squares added in chunk order) travels with the last chunk; then release `epoch` into
 * flag_peers[q][rank] for every q.  One call at a time per device (the side streams are
 * shared).  Rowwise split only; TG_FLAG_INDEX32 as for tg_power_step_f64. */
TG_API int tg_power_step_ce_f64(const tg_csr* A, const double* x, int32_t nparts, int32_t rank, int64_t stride,
                                double* const* y_peers, uint64_t* const* flag_peers, uint64_t epoch, int32_t nchunks,
                                const tg_sched* s, void* workspace, size_t workspace_bytes, tg_stream_t stream);
/* Copies the power workspace's error word to *err (synchronises `stream`): 16 = a peer
 * wait ran out.  Zero when nothing went wrong. */
TG_API int tg_power_error(const void* workspace, uint32_t* err, tg_stream_t stream);
/* Clears the power workspace's error word (asynchronously on `stream`). */
TG_API int tg_power_clear_error(void* workspace, tg_stream_t stream);
/* Bounded wait (2 s) until every entry of this rank's flag array reached `epoch`: the
 * pushes of the last step have landed and the local iterate is complete.  Returns at once
 * (error word unchanged) when the workspace's error word is already set. */
TG_API int tg_p2p_wait(const uint64_t* flag_local, int32_t nparts, uint64_t epoch, void* workspace,
                       size_t workspace_bytes, tg_stream_t stream);

/* Exchange buffers of the fused step: device memory from cudaMalloc (zero-filled), so
 * that a CUDA IPC handle maps the buffer itself.  tg_ipc_open maps a peer's buffer into
 * the current device's context with lazy peer access; close it before the owner frees. */
TG_API int tg_peer_buffer_alloc(size_t bytes, void** ptr);
TG_API int tg_peer_buffer_free(void* ptr);
TG_API int tg_ipc_get_handle(const void* ptr, void* handle /* 64 bytes */);
TG_API int tg_ipc_open(const void* handle /* 64 bytes */, void** ptr);
TG_API int tg_ipc_close(void* ptr);

/* ------------------------------------------- column-locality reordering (new) */
/* Reverse Cuthill-McKee order of a square matrix (no counterpart in the reference; an
 * optional preprocessing pass).  HOST arrays: indptr[n+1], indices[indptr[n]] in [0, n).
 * perm[new] = old, a permutation of 0..n-1 computed on the symmetrised pattern
 * (A + A^T).  Applying it as A' = P A P^T, x' = P x (B' = P B, V' = P V, U' = P U) gives
 * y' = P y: rows that share columns get nearby numbers, which raises the L2 hit rate of
 * the gathers where the pattern has such structure. */
TG_API int tg_rcm_order(int64_t n, const int64_t* indptr, const int64_t* indices, int64_t* perm);

/* ----------------------------------------------- SpMV that allocates nothing */
/* No counterpart in the reference.  y = A x (fp64, merge split) for callers that can
 * pass only inputs and outputs -- a host that owns the whole GPU memory pool, or a path
 * that cannot afford cudaMalloc's implicit synchronisation.  Its scratch is a fixed
 * 1 MiB array in the library's device memory (on every GPU that loads the library,
 * until the process exits), so there is no workspace argument and nothing is allocated.
 * Limit: the partition of A's nonzeros must fit the array -- about 67 million nonzeros
 * with block_size 256, 33 million with 128; larger calls return TG_EINVAL naming the
 * limit.  The schedule is resolved as for tg_spmv_f64 (NULL: the tg_set_schedule one),
 * with the merge split forced.  The first call on a device looks up the array's address
 * (cudaGetSymbolAddress) and should come before any stream capture there; the address is
 * cached for the process and does not survive cudaDeviceReset.  All calls share the array,
 * so calls that overlap on the GPU race: order them on one stream.  Bounds checking and
 * plan reuse are not available here. */
TG_API int tg_spmv_f64_noalloc(const tg_csr* A, const double* x, double* y, const tg_sched* s,
                               tg_stream_t stream);

/* ------------------------------------------------- multi-GPU, one process (new) */
/* One process driving `nranks` GPUs of a node (no counterpart in the reference; the
 * multi-GPU mode of north_star).  tg_dist_init creates a stream per GPU and enables peer
 * access between every pair (TG_EUNSUPPORTED when a pair cannot map each other's
 * memory); one rank per GPU, each device listed once, at most 8.  The calls take HOST
 * CSR matrices and host dense operands, split the rows into nnz-balanced contiguous
 * shards, replicate the dense inputs, run every shard on its GPU and gather the output
 * rows to the host.  timeout_s > 0 is a host deadline: past it the call returns
 * TG_ETIMEDOUT, after the device work (whose own waits are bounded) has stopped.
 * The caller's current device is left unchanged. */
typedef struct tg_dist tg_dist;
TG_API int tg_dist_init(int32_t nranks, const int32_t* devices, tg_dist** out);
/* Waits for the context's work and releases it (NULL is accepted). */
TG_API int tg_dist_finalize(tg_dist* d);
/* `iters` power iterations x <- A x / ||A x|| of a square fp64 matrix from x0 (host, A.cols
 * values, any scale) with the fused step + peer-memory exchange; x_out (host, A.rows)
 * receives the final iterate, *lambda the norm of the last A x (x0 normalised and its
 * norm when iters = 0).  A peer that stops answering ends the call with TG_ETIMEDOUT. */
TG_API int tg_dist_spmv_power(tg_dist* d, const tg_csr* A, const double* x0, int32_t iters, const tg_sched* s,
                              double* x_out, double* lambda, double timeout_s);
/* C (host, A.rows x k) = A B with A's values fp32 and B (host, A.cols x k) fp32. */
TG_API int tg_dist_spmm_f32(tg_dist* d, const tg_csr* A, const float* B, int64_t k, float* C, const tg_sched* s,
                            double timeout_s);
/* out (host, A.nnz, A's order) = A .* (U V^T) on A's pattern; U (A.rows x k), V (A.cols x k). */
TG_API int tg_dist_sddmm_f32(tg_dist* d, const tg_csr* A, const float* U, const float* V, int64_t k, float* out,
                             const tg_sched* s, double timeout_s);

/* --------------------------------------------- reference-compatible launchers */
/* Signatures as emitted by tilegen/codegen.py:_abi (226-280) for the standard kernels
 * of tilegen/dsl.py:214-256; argument order/meaning as in tilegen/verify.py:166-173. */
TG_API void launch_spmv(const int64_t* indptr, const int64_t* indices, const double* data,
                 const double* x, double* y, int64_t M, int64_t N, int64_t nnz);
TG_API void launch_spmm(const int64_t* indptr, const int64_t* indices, const double* data,
                 const double* B, double* C, int64_t M, int64_t N, int64_t K, int64_t nnz);
TG_API void launch_sddmm(const int64_t* indptr, const int64_t* indices, const double* data,
                  const double* U, const double* V, double* C, int64_t M, int64_t N,
                  int64_t K, int64_t nnz);
TG_API void launch_fused_spmv_axpy(const int64_t* indptr, const int64_t* indices,
                            const double* data, const double* x, const double* w, double* z,
                            double alpha, double beta, int64_t M, int64_t N, int64_t nnz);
TG_API void launch_axpy(const double* x, const double* w, double* z, double alpha, double beta,
                 int64_t M);

#ifdef __cplusplus
}
#endif

#endif /* TILEGEN_B200_H */
