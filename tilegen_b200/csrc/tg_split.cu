// Streaming partition pass of the merge-split kernels (see tg_split.cuh).
#include "tg_split.cuh"

namespace tg {

__global__ void partition_kernel(const int64_t* __restrict__ indptr, int64_t rows, int64_t S, int64_t nchunks,
                                 int64_t* __restrict__ own_first, int* __restrict__ cnt, uint32_t* err) {
    pdl_trigger();
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    for (int64_t r = tid; r <= rows; r += stride) {
        const int64_t hi = indptr[r];
        // chunks c with lo < c*S <= hi: c0 = smallest c with c*S > lo, c1 = hi / S
        int64_t c0 = 0;
        if (r > 0) c0 = indptr[r - 1] / S + 1;
        int64_t c1 = hi / S;
        if (c1 > nchunks - 1) c1 = nchunks - 1;
        for (int64_t c = c0; c <= c1; ++c) own_first[c] = r;
    }
    if (cnt)
        for (int64_t c = tid; c < nchunks; c += stride) cnt[c] = 0;
    if (tid == 0) {
        own_first[nchunks] = rows;
        if (err) *err = 0u;
    }
}

int launch_partition(const int64_t* indptr, int64_t rows, int64_t nnz, int64_t S, const SplitWs& ws,
                     cudaStream_t stream) {
    const int64_t nchunks = ceil_div(nnz, S);
    const int threads = 256;
    int64_t blocks = ceil_div(rows + 1, threads);
    if (blocks > 148 * 16) blocks = 148 * 16;
    if (blocks < 1) blocks = 1;
    partition_kernel<<<(unsigned)blocks, threads, 0, stream>>>(indptr, rows, S, nchunks, ws.own_first, ws.cnt,
                                                               ws.err);
    return check_launch("partition_kernel");
}

}  // namespace tg
