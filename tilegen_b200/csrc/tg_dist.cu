// tg_dist_*: the multi-GPU entry points of the C ABI, for one process driving several
// GPUs of a node (no counterpart in the reference; north_star's multi-GPU mode).
//
// A tg_dist context holds one stream per GPU and has peer access enabled between every
// pair.  Each call takes a HOST CSR matrix and host dense operands, splits the rows into
// nnz-balanced contiguous shards (rank r gets rows [b[r], b[r+1]), b[r] = first row whose
// nonzero offset reaches r * nnz / nranks), uploads each shard with the dense inputs
// replicated, runs the shard on its GPU, and gathers the output rows back to the host.
//
//  * tg_dist_spmv_power: the power iteration with the fused step + exchange kernel of
//    tg_power.cu (power_p2p_kernel): every GPU stores its finished rows straight into
//    every GPU's next iterate through peer pointers and releases a per-rank epoch flag;
//    the next step waits (bounded, 2 s) on all flags.  Kernels of different ranks wait
//    on one another only across GPUs: one rank per GPU, never two on one GPU.
//  * tg_dist_spmm_f32 / tg_dist_sddmm_f32: row shards, no communication.
//
// Every call honours a host deadline (timeout_s > 0): it returns TG_ETIMEDOUT when the
// device work has not finished by then.  It still waits for that work to stop before
// freeing the shard buffers (every device-side wait is bounded), so no kernel ever runs
// on freed memory.  The caller's current device is restored on return.
#include <algorithm>
#include <chrono>
#include <cstring>
#include <vector>

#include "tg_common.cuh"

namespace tg {
size_t power_ws_bytes(int64_t nnz, const tg_sched& s);
int shard_norm2_run(double* shard, int64_t rows, int64_t stride, void* ws, size_t ws_bytes, cudaStream_t st);
int power_finalize_run(const double* x, int nparts, int64_t stride, int part, int64_t rows, double* x_out,
                       double* lambda_out, cudaStream_t st);
int power_step_p2p_run(const tg_csr& A, const double* x, int nparts, int rank, int64_t stride,
                       double* const* y_peers, unsigned long long* const* flag_peers, unsigned long long epoch,
                       const tg_sched& s, void* ws, size_t ws_bytes, cudaStream_t st);
size_t power_err_offset();
int p2p_wait_run(const unsigned long long* flag_local, int nparts, unsigned long long epoch, void* ws,
                 size_t ws_bytes, cudaStream_t st);
template <typename T>
size_t dense_ws_bytes(int64_t rows, int64_t nnz, int64_t K, const tg_sched& s, bool is_spmm);
template <typename T>
int dense_run(bool is_spmm, const tg_csr& A, const T* B, const T* U, T* C, int64_t K, const tg_sched& s, void* ws,
              size_t ws_bytes, cudaStream_t st);
}  // namespace tg

extern "C" int tg_renumber_columns(const int64_t* indices, int64_t* out, int64_t nnz, const int64_t* bounds,
                                   int32_t nparts, int64_t stride, tg_stream_t stream);

using namespace tg;

struct tg_dist {
    int n = 0;
    std::vector<int> dev;
    std::vector<cudaStream_t> st;
};

namespace {

constexpr int kMaxRanks = 8;  // the fused exchange kernel's peer table

// Restores the caller's current device when the call returns.
struct DeviceGuard {
    int saved = 0;
    bool ok = false;
    DeviceGuard() { ok = cudaGetDevice(&saved) == cudaSuccess; }
    ~DeviceGuard() {
        if (ok) cudaSetDevice(saved);
    }
};

// Device allocations of one call, freed (after all streams are idle) when it returns.
struct Allocs {
    std::vector<std::pair<int, void*>> p;
    int get(int dev, size_t bytes, void** out, bool zero) {
        *out = nullptr;
        int rc = check_cuda(cudaSetDevice(dev), "cudaSetDevice");
        if (rc != TG_OK) return rc;
        rc = check_cuda(cudaMalloc(out, std::max<size_t>(bytes, 16)), "cudaMalloc");
        if (rc != TG_OK) return rc;
        p.emplace_back(dev, *out);
        if (zero) return check_cuda(cudaMemset(*out, 0, std::max<size_t>(bytes, 16)), "cudaMemset");
        return TG_OK;
    }
    ~Allocs() {
        // nothing queued by this call may still use the buffers (error paths return early)
        std::vector<int> devs;
        for (auto& q : p)
            if (std::find(devs.begin(), devs.end(), q.first) == devs.end()) devs.push_back(q.first);
        for (int dv : devs) {
            cudaSetDevice(dv);
            cudaDeviceSynchronize();
        }
        for (auto& q : p) {
            cudaSetDevice(q.first);
            cudaFree(q.second);
        }
    }
};

int sync_all(tg_dist* d) {
    int rc = TG_OK;
    for (int r = 0; r < d->n; ++r) {
        cudaSetDevice(d->dev[r]);
        const int e = check_cuda(cudaStreamSynchronize(d->st[r]), "cudaStreamSynchronize");
        if (rc == TG_OK) rc = e;
    }
    return rc;
}

// Waits until every rank's stream is idle or the deadline passes (timeout_s <= 0: no
// deadline).  Returns TG_ETIMEDOUT past the deadline after waiting for the work to stop.
int wait_deadline(tg_dist* d, double timeout_s) {
    if (timeout_s > 0.0) {
        const auto t0 = std::chrono::steady_clock::now();
        for (;;) {
            bool busy = false;
            for (int r = 0; r < d->n; ++r) {
                cudaSetDevice(d->dev[r]);
                const cudaError_t e = cudaStreamQuery(d->st[r]);
                if (e == cudaErrorNotReady) {
                    busy = true;
                } else if (e != cudaSuccess) {
                    return check_cuda(e, "cudaStreamQuery");
                }
            }
            if (!busy) break;
            const double dt = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
            if (dt > timeout_s) {
                sync_all(d);  // bounded device waits: the work stops by itself
                return set_error(TG_ETIMEDOUT, "tg_dist: device work did not finish within %.3f s", timeout_s);
            }
        }
    }
    return sync_all(d);
}

int fill_sched(const tg_sched* s, tg_sched* out) {
    tg_sched c;
    if (s) {
        c = *s;
    } else {
        tg_default_schedule(&c);
    }
    if (c.tile <= 0) c.tile = 32;
    if (c.threads_per_row <= 0) c.threads_per_row = 1;
    if (c.unroll <= 0) c.unroll = 1;
    if (c.vector_width <= 0) c.vector_width = 1;
    if (c.block_size <= 0) c.block_size = 128;
    if (c.split == TG_SPLIT_AUTO) c.split = TG_SPLIT_MERGE;
    const int rc = tg_validate_schedule(&c);
    if (rc != TG_OK) return rc;
    *out = c;
    return TG_OK;
}

int check_host_csr(const tg_csr* A, const char* op) {
    if (!A) return set_error(TG_EINVAL, "%s: null CSR descriptor", op);
    if (A->rows < 0 || A->cols < 0 || A->nnz < 0) return set_error(TG_EINVAL, "%s: negative size", op);
    if (!A->indptr || (A->nnz > 0 && (!A->indices || !A->data))) return set_error(TG_EINVAL, "%s: null array", op);
    if (A->indptr[0] != 0 || A->indptr[A->rows] != A->nnz)
        return set_error(TG_EINVAL, "%s: indptr must start at 0 and end at nnz", op);
    for (int64_t i = 0; i < A->rows; ++i)
        if (A->indptr[i + 1] < A->indptr[i]) return set_error(TG_EINVAL, "%s: indptr decreases at row %lld", op,
                                                              (long long)i);
    return TG_OK;
}

// nnz-balanced row bounds: b[r] = first row whose offset reaches r * nnz / n.
std::vector<int64_t> row_bounds(const tg_csr* A, int n) {
    std::vector<int64_t> b(n + 1, 0);
    b[n] = A->rows;
    for (int r = 1; r < n; ++r) {
        const int64_t target = (int64_t)((__int128)r * A->nnz / n);
        b[r] = std::lower_bound(A->indptr, A->indptr + A->rows + 1, target) - A->indptr;
        b[r] = std::max(b[r], b[r - 1]);
    }
    return b;
}

struct Shard {
    int64_t r0 = 0, r1 = 0, p0 = 0, nnz = 0;
    int64_t* indptr = nullptr;
    int64_t* indices = nullptr;
    void* data = nullptr;
};

// Uploads rank r's rows (indptr rebased to 0) to its GPU.
int upload_shard(tg_dist* d, int r, const tg_csr* A, const std::vector<int64_t>& b, size_t elem, Allocs& al,
                 Shard* s) {
    s->r0 = b[r];
    s->r1 = b[r + 1];
    s->p0 = A->indptr[s->r0];
    s->nnz = A->indptr[s->r1] - s->p0;
    const int64_t rows = s->r1 - s->r0;
    std::vector<int64_t> ip(rows + 1);
    for (int64_t i = 0; i <= rows; ++i) ip[i] = A->indptr[s->r0 + i] - s->p0;
    int rc = al.get(d->dev[r], sizeof(int64_t) * (rows + 1), (void**)&s->indptr, false);
    if (rc == TG_OK) rc = al.get(d->dev[r], sizeof(int64_t) * s->nnz, (void**)&s->indices, false);
    if (rc == TG_OK) rc = al.get(d->dev[r], elem * s->nnz, &s->data, false);
    if (rc != TG_OK) return rc;
    // synchronous copies: ip is a temporary
    rc = check_cuda(cudaMemcpy(s->indptr, ip.data(), sizeof(int64_t) * (rows + 1), cudaMemcpyHostToDevice), "H2D");
    if (rc == TG_OK && s->nnz > 0)
        rc = check_cuda(cudaMemcpy(s->indices, A->indices + s->p0, sizeof(int64_t) * s->nnz, cudaMemcpyHostToDevice),
                        "H2D");
    if (rc == TG_OK && s->nnz > 0)
        rc = check_cuda(cudaMemcpy(s->data, static_cast<const char*>(A->data) + elem * s->p0, elem * s->nnz,
                                   cudaMemcpyHostToDevice),
                        "H2D");
    return rc;
}

}  // namespace

extern "C" {

int tg_dist_init(int32_t nranks, const int32_t* devices, tg_dist** out) {
    if (!out) return set_error(TG_EINVAL, "tg_dist_init: null output pointer");
    *out = nullptr;
    if (nranks < 1 || nranks > kMaxRanks || !devices)
        return set_error(TG_EINVAL, "tg_dist_init: need 1..%d ranks and a device list (got %d)", kMaxRanks, nranks);
    for (int i = 0; i < nranks; ++i)
        for (int j = 0; j < i; ++j)
            if (devices[i] == devices[j])
                return set_error(TG_EINVAL, "tg_dist_init: device %d listed twice (one rank per GPU)", devices[i]);
    int count = 0;
    int rc = check_cuda(cudaGetDeviceCount(&count), "cudaGetDeviceCount");
    if (rc != TG_OK) return rc;
    for (int i = 0; i < nranks; ++i)
        if (devices[i] < 0 || devices[i] >= count)
            return set_error(TG_EINVAL, "tg_dist_init: device %d does not exist (%d visible)", devices[i], count);
    DeviceGuard guard;
    tg_dist* d = new tg_dist();
    d->n = nranks;
    d->dev.assign(devices, devices + nranks);
    for (int r = 0; r < nranks; ++r) {
        cudaStream_t s = nullptr;
        rc = check_cuda(cudaSetDevice(devices[r]), "cudaSetDevice");
        if (rc == TG_OK) rc = check_cuda(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking), "cudaStreamCreate");
        if (rc != TG_OK) {
            tg_dist_finalize(d);
            return rc;
        }
        d->st.push_back(s);
    }
    for (int r = 0; r < nranks && rc == TG_OK; ++r) {
        cudaSetDevice(devices[r]);
        for (int q = 0; q < nranks && rc == TG_OK; ++q) {
            if (q == r) continue;
            int can = 0;
            rc = check_cuda(cudaDeviceCanAccessPeer(&can, devices[r], devices[q]), "cudaDeviceCanAccessPeer");
            if (rc == TG_OK && !can)
                rc = set_error(TG_EUNSUPPORTED, "tg_dist_init: GPU %d cannot map GPU %d's memory", devices[r],
                               devices[q]);
            if (rc == TG_OK) {
                const cudaError_t e = cudaDeviceEnablePeerAccess(devices[q], 0);
                if (e == cudaErrorPeerAccessAlreadyEnabled)
                    cudaGetLastError();  // clear it: enabled earlier in this process
                else
                    rc = check_cuda(e, "cudaDeviceEnablePeerAccess");
            }
        }
    }
    if (rc != TG_OK) {
        tg_dist_finalize(d);
        return rc;
    }
    *out = d;
    return TG_OK;
}

int tg_dist_finalize(tg_dist* d) {
    if (!d) return TG_OK;
    DeviceGuard guard;
    int rc = TG_OK;
    for (size_t r = 0; r < d->st.size(); ++r) {
        cudaSetDevice(d->dev[r]);
        const int e = check_cuda(cudaStreamSynchronize(d->st[r]), "cudaStreamSynchronize");
        cudaStreamDestroy(d->st[r]);
        if (rc == TG_OK) rc = e;
    }
    delete d;
    return rc;
}

int tg_dist_spmv_power(tg_dist* d, const tg_csr* A, const double* x0, int32_t iters, const tg_sched* s,
                       double* x_out, double* lambda, double timeout_s) {
    if (!d) return set_error(TG_EINVAL, "tg_dist_spmv_power: null context");
    int rc = check_host_csr(A, "tg_dist_spmv_power");
    if (rc != TG_OK) return rc;
    if (A->rows != A->cols) return set_error(TG_EINVAL, "tg_dist_spmv_power: the matrix must be square");
    if (iters < 0 || (A->rows > 0 && (!x0 || !x_out)) || !lambda)
        return set_error(TG_EINVAL, "tg_dist_spmv_power: bad iters or null x0/x_out/lambda");
    for (int64_t p = 0; p < A->nnz; ++p)
        if (A->indices[p] < 0 || A->indices[p] >= A->cols)
            return set_error(TG_EBOUNDS, "tg_dist_spmv_power: column index out of range at %lld", (long long)p);
    tg_sched sc;
    rc = fill_sched(s, &sc);
    if (rc != TG_OK) return rc;
    sc.split = TG_SPLIT_ROWWISE;  // the fused exchange kernel is rowwise
    DeviceGuard guard;
    const int n = d->n;
    const std::vector<int64_t> b = row_bounds(A, n);
    int64_t longest = 0;
    for (int r = 0; r < n; ++r) longest = std::max(longest, b[r + 1] - b[r]);
    const int64_t stride = ((longest + 1 + 31) / 32) * 32;
    const int64_t xlen = (int64_t)n * stride;

    Allocs al;
    std::vector<Shard> sh(n);
    std::vector<double*> xb0(n), xb1(n), xo(n), lam(n);
    std::vector<unsigned long long*> flags(n);
    std::vector<void*> ws(n);
    std::vector<size_t> wsb(n);
    for (int r = 0; r < n && rc == TG_OK; ++r) {
        rc = upload_shard(d, r, A, b, sizeof(double), al, &sh[r]);
        if (rc == TG_OK) rc = check_cuda(cudaSetDevice(d->dev[r]), "cudaSetDevice");
        if (rc == TG_OK && sh[r].nnz > 0)  // columns to the padded layout, in place
            rc = tg_renumber_columns(sh[r].indices, sh[r].indices, sh[r].nnz, b.data(), n, stride, d->st[r]);
        if (rc == TG_OK) rc = al.get(d->dev[r], sizeof(double) * xlen, (void**)&xb0[r], true);
        if (rc == TG_OK) rc = al.get(d->dev[r], sizeof(double) * xlen, (void**)&xb1[r], true);
        if (rc == TG_OK) rc = al.get(d->dev[r], sizeof(double) * (b[r + 1] - b[r]), (void**)&xo[r], false);
        if (rc == TG_OK) rc = al.get(d->dev[r], sizeof(double), (void**)&lam[r], false);
        if (rc == TG_OK) rc = al.get(d->dev[r], sizeof(unsigned long long) * n, (void**)&flags[r], true);
        wsb[r] = power_ws_bytes(sh[r].nnz, sc);
        if (rc == TG_OK) rc = al.get(d->dev[r], wsb[r], &ws[r], true);
    }
    if (rc != TG_OK) return rc;

    // x0: every rank's shard and its slot, then every shard (with its slot) to every rank
    for (int r = 0; r < n && rc == TG_OK; ++r) {
        cudaSetDevice(d->dev[r]);
        const int64_t rows = b[r + 1] - b[r];
        double* own = xb0[r] + (int64_t)r * stride;
        if (rows > 0)
            rc = check_cuda(cudaMemcpyAsync(own, x0 + b[r], sizeof(double) * rows, cudaMemcpyHostToDevice, d->st[r]),
                            "H2D x0");
        if (rc == TG_OK) rc = shard_norm2_run(own, rows, stride, ws[r], wsb[r], d->st[r]);
    }
    if (rc == TG_OK) rc = sync_all(d);
    for (int r = 0; r < n && rc == TG_OK; ++r) {
        cudaSetDevice(d->dev[r]);
        for (int q = 0; q < n && rc == TG_OK; ++q)
            if (q != r)
                rc = check_cuda(cudaMemcpyPeerAsync(xb0[r] + (int64_t)q * stride, d->dev[r],
                                                    xb0[q] + (int64_t)q * stride, d->dev[q], sizeof(double) * stride,
                                                    d->st[r]),
                                "cudaMemcpyPeerAsync");
    }
    if (rc == TG_OK) rc = sync_all(d);
    if (rc != TG_OK) return rc;

    // iterations: epoch e reads buffer (e-1)%2 and writes the other on every rank
    for (int32_t e = 1; e <= iters && rc == TG_OK; ++e) {
        const bool even = (e % 2) == 1;  // epoch 1 reads xb0
        double* ypeer[kMaxRanks];
        unsigned long long* fpeer[kMaxRanks];
        for (int q = 0; q < n; ++q) {
            ypeer[q] = even ? xb1[q] : xb0[q];
            fpeer[q] = flags[q];
        }
        for (int r = 0; r < n && rc == TG_OK; ++r) {
            cudaSetDevice(d->dev[r]);
            const tg_csr Ar{b[r + 1] - b[r], xlen, sh[r].nnz, sh[r].indptr, sh[r].indices, sh[r].data};
            rc = power_step_p2p_run(Ar, even ? xb0[r] : xb1[r], n, r, stride, ypeer, fpeer,
                                    (unsigned long long)e, sc, ws[r], wsb[r], d->st[r]);
        }
    }
    const bool final_in_xb0 = (iters % 2) == 0;
    for (int r = 0; r < n && rc == TG_OK; ++r) {
        cudaSetDevice(d->dev[r]);
        if (iters > 0) rc = p2p_wait_run(flags[r], n, (unsigned long long)iters, ws[r], wsb[r], d->st[r]);
        if (rc == TG_OK)
            rc = power_finalize_run(final_in_xb0 ? xb0[r] : xb1[r], n, stride, r, b[r + 1] - b[r], xo[r], lam[r],
                                    d->st[r]);
    }
    const int wrc = wait_deadline(d, timeout_s);  // always wait: the buffers are freed on return
    if (rc == TG_OK) rc = wrc;
    if (rc != TG_OK) return rc;
    for (int r = 0; r < n && rc == TG_OK; ++r) {
        cudaSetDevice(d->dev[r]);
        uint32_t err = 0;
        rc = check_cuda(cudaMemcpy(&err, static_cast<char*>(ws[r]) + power_err_offset(), sizeof(uint32_t),
                                   cudaMemcpyDeviceToHost),
                        "D2H error word");
        if (rc == TG_OK && err)
            rc = set_error(TG_ETIMEDOUT, "tg_dist_spmv_power: rank %d gave up waiting for its peers (error 0x%x)", r,
                           err);
        const int64_t rows = b[r + 1] - b[r];
        if (rc == TG_OK && rows > 0)
            rc = check_cuda(cudaMemcpy(x_out + b[r], xo[r], sizeof(double) * rows, cudaMemcpyDeviceToHost), "D2H x");
        if (rc == TG_OK && r == 0)
            rc = check_cuda(cudaMemcpy(lambda, lam[0], sizeof(double), cudaMemcpyDeviceToHost), "D2H lambda");
    }
    return rc;
}

static int dist_dense(tg_dist* d, bool is_spmm, const tg_csr* A, const float* BV, const float* U, int64_t K,
                      float* out, const tg_sched* s, double timeout_s, const char* op) {
    if (!d) return set_error(TG_EINVAL, "%s: null context", op);
    int rc = check_host_csr(A, op);
    if (rc != TG_OK) return rc;
    if (K < 1) return set_error(TG_EINVAL, "%s: K must be >= 1", op);
    if (A->nnz > 0 && (!BV || !out || (!is_spmm && !U))) return set_error(TG_EINVAL, "%s: null dense operand", op);
    if (is_spmm && A->rows > 0 && !out) return set_error(TG_EINVAL, "%s: null C", op);
    for (int64_t p = 0; p < A->nnz; ++p)
        if (A->indices[p] < 0 || A->indices[p] >= A->cols)
            return set_error(TG_EBOUNDS, "%s: column index out of range at %lld", op, (long long)p);
    tg_sched sc;
    rc = fill_sched(s, &sc);
    if (rc != TG_OK) return rc;
    DeviceGuard guard;
    const int n = d->n;
    const std::vector<int64_t> b = row_bounds(A, n);
    Allocs al;
    std::vector<Shard> sh(n);
    std::vector<float*> dB(n), dU(n), dO(n);
    std::vector<void*> ws(n);
    std::vector<size_t> wsb(n);
    const size_t full = sizeof(float) * (size_t)A->cols * (size_t)K;
    for (int r = 0; r < n && rc == TG_OK; ++r) {
        rc = upload_shard(d, r, A, b, sizeof(float), al, &sh[r]);
        const int64_t rows = b[r + 1] - b[r];
        if (rc == TG_OK) rc = al.get(d->dev[r], full, (void**)&dB[r], false);
        if (rc == TG_OK && A->cols > 0)
            rc = check_cuda(cudaMemcpyAsync(dB[r], BV, full, cudaMemcpyHostToDevice, d->st[r]), "H2D B/V");
        if (rc == TG_OK && !is_spmm) {
            rc = al.get(d->dev[r], sizeof(float) * rows * K, (void**)&dU[r], false);
            if (rc == TG_OK && rows > 0)
                rc = check_cuda(cudaMemcpyAsync(dU[r], U + b[r] * K, sizeof(float) * rows * K, cudaMemcpyHostToDevice,
                                                d->st[r]),
                                "H2D U");
        }
        const size_t out_n = is_spmm ? (size_t)rows * K : (size_t)sh[r].nnz;
        if (rc == TG_OK) rc = al.get(d->dev[r], sizeof(float) * out_n, (void**)&dO[r], false);
        wsb[r] = dense_ws_bytes<float>(rows, sh[r].nnz, K, sc, is_spmm);
        if (rc == TG_OK) rc = al.get(d->dev[r], wsb[r], &ws[r], true);
        if (rc == TG_OK) rc = check_cuda(cudaSetDevice(d->dev[r]), "cudaSetDevice");
        if (rc == TG_OK) {
            const tg_csr Ar{rows, A->cols, sh[r].nnz, sh[r].indptr, sh[r].indices, sh[r].data};
            rc = dense_run<float>(is_spmm, Ar, dB[r], dU[r], dO[r], K, sc, ws[r], wsb[r], d->st[r]);
        }
    }
    const int wrc = wait_deadline(d, timeout_s);
    if (rc == TG_OK) rc = wrc;
    for (int r = 0; r < n && rc == TG_OK; ++r) {
        cudaSetDevice(d->dev[r]);
        const int64_t rows = b[r + 1] - b[r];
        if (is_spmm && rows > 0)
            rc = check_cuda(cudaMemcpy(out + b[r] * K, dO[r], sizeof(float) * rows * K, cudaMemcpyDeviceToHost),
                            "D2H C");
        if (!is_spmm && sh[r].nnz > 0)
            rc = check_cuda(cudaMemcpy(out + sh[r].p0, dO[r], sizeof(float) * sh[r].nnz, cudaMemcpyDeviceToHost),
                            "D2H out");
    }
    return rc;
}

int tg_dist_spmm_f32(tg_dist* d, const tg_csr* A, const float* B, int64_t k, float* C, const tg_sched* s,
                     double timeout_s) {
    return dist_dense(d, true, A, B, nullptr, k, C, s, timeout_s, "tg_dist_spmm_f32");
}

int tg_dist_sddmm_f32(tg_dist* d, const tg_csr* A, const float* U, const float* V, int64_t k, float* out,
                      const tg_sched* s, double timeout_s) {
    return dist_dense(d, false, A, V, U, k, out, s, timeout_s, "tg_dist_sddmm_f32");
}

}  // extern "C"
