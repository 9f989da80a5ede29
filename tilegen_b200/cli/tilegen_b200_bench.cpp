// tilegen_b200_bench: the b200 counterpart of the reference's C++ harness
// (cpp/src/harness.cpp:117-268, `tilegen_bench`).
//
// Same command line and JSON result line: loads a CSR matrix from a TGM1 file (the
// little-endian dump of tilegen/matrices.py:38-46, 240-252), dlopen()s a library that
// exports the reference ABI `launch_<kernel>` (libtilegen_b200.so by default, or any
// CUDA object the reference's code generator emitted), runs the kernel, times it and
// checks it against a host evaluation of the same formula.  The differences are the
// ones a GPU needs: operands live in device memory (copied once, outside the timed
// region, like tilegen/verify.py:103-163 does for the cuda backend) and every call is
// timed with CUDA events.  When the library also exports tg_set_schedule, the schedule
// knobs (--tile --tpr --unroll --vec --block --split) are applied first.
//
//   tilegen_b200_bench --kernel K --matrix M.bin [--lib L.so] [--config JSON]
//                      [--iters N] [--warmup N] [--K 32] [schedule knobs]
#include <cuda_runtime.h>
#include <dlfcn.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <iostream>
#include <sstream>
#include <string>
#include <vector>

#include "../../include/tilegen_b200.h"

namespace {

constexpr uint32_t kTgm1Magic = 0x54474D31u;  // "TGM1"

struct Matrix {
    int64_t rows = 0, cols = 0, nnz = 0;
    std::vector<int64_t> indptr, indices;
    std::vector<double> data;
};

[[noreturn]] void die(int code, const std::string& msg) {
    std::cerr << "error: " << msg << "\n";
    std::exit(code);
}

Matrix load_tgm1(const std::string& path) {
    std::ifstream fh(path, std::ios::binary);
    if (!fh) die(2, "cannot open matrix " + path);
    uint32_t magic = 0;
    Matrix m;
    fh.read(reinterpret_cast<char*>(&magic), 4);
    fh.read(reinterpret_cast<char*>(&m.rows), 8);
    fh.read(reinterpret_cast<char*>(&m.cols), 8);
    fh.read(reinterpret_cast<char*>(&m.nnz), 8);
    if (!fh || magic != kTgm1Magic) die(2, path + ": not a TGM1 file");
    if (m.rows < 0 || m.cols < 0 || m.nnz < 0) die(2, path + ": negative header field");
    m.indptr.resize(m.rows + 1);
    m.indices.resize(m.nnz);
    m.data.resize(m.nnz);
    fh.read(reinterpret_cast<char*>(m.indptr.data()), 8 * (m.rows + 1));
    fh.read(reinterpret_cast<char*>(m.indices.data()), 8 * m.nnz);
    fh.read(reinterpret_cast<char*>(m.data.data()), 8 * m.nnz);
    if (!fh) die(2, path + ": truncated TGM1 file");
    if (m.indptr[0] != 0 || m.indptr[m.rows] != m.nnz) die(2, path + ": inconsistent indptr");
    for (int64_t i = 0; i < m.rows; ++i)
        if (m.indptr[i + 1] < m.indptr[i]) die(2, path + ": indptr not monotone");
    for (int64_t p = 0; p < m.nnz; ++p)
        if (m.indices[p] < 0 || m.indices[p] >= m.cols) die(2, path + ": column index out of range");
    return m;
}

struct Args {
    std::string kernel, matrix, lib, config = "{}", split;
    int iters = 20, warmup = 3;
    int64_t K = 32;
    int tile = 0, tpr = 0, unroll = 0, vec = 0, block = 0;
};

Args parse(int argc, char** argv) {
    Args a;
    for (int i = 1; i < argc; ++i) {
        const std::string k = argv[i];
        auto next = [&]() -> std::string {
            if (i + 1 >= argc) die(2, "missing value for " + k);
            return argv[++i];
        };
        if (k == "--kernel") a.kernel = next();
        else if (k == "--matrix") a.matrix = next();
        else if (k == "--lib") a.lib = next();
        else if (k == "--config") a.config = next();
        else if (k == "--backend") next();  // accepted for the reference's command line; always cuda
        else if (k == "--iters") a.iters = std::atoi(next().c_str());
        else if (k == "--warmup") a.warmup = std::atoi(next().c_str());
        else if (k == "--K") a.K = std::atoll(next().c_str());
        else if (k == "--tile") a.tile = std::atoi(next().c_str());
        else if (k == "--tpr") a.tpr = std::atoi(next().c_str());
        else if (k == "--unroll") a.unroll = std::atoi(next().c_str());
        else if (k == "--vec") a.vec = std::atoi(next().c_str());
        else if (k == "--block") a.block = std::atoi(next().c_str());
        else if (k == "--split") a.split = next();
        else die(2, "unknown argument " + k);
    }
    if (a.iters < 1 || a.warmup < 0 || a.K < 1) die(2, "bad --iters/--warmup/--K");
    return a;
}

std::string default_lib(const char* argv0) {
    std::string self = argv0;
    const size_t slash = self.rfind('/');
    return (slash == std::string::npos ? std::string(".") : self.substr(0, slash)) + "/libtilegen_b200.so";
}

void check(cudaError_t e, const char* what) {
    if (e != cudaSuccess) die(4, std::string(what) + ": " + cudaGetErrorString(e));
}

template <typename T>
T* to_device(const std::vector<T>& h) {
    T* d = nullptr;
    check(cudaMalloc(&d, std::max<size_t>(h.size(), 1) * sizeof(T)), "cudaMalloc");
    if (!h.empty()) check(cudaMemcpy(d, h.data(), h.size() * sizeof(T), cudaMemcpyHostToDevice), "cudaMemcpy H2D");
    return d;
}

std::string json_escape(const std::string& s) {
    std::string o;
    for (char c : s) {
        if (c == '"' || c == '\\') o += '\\';
        o += c;
    }
    return o;
}

}  // namespace

int main(int argc, char** argv) {
    Args args = parse(argc, argv);
    if (args.kernel.empty() || args.matrix.empty()) {
        std::cerr << "usage: tilegen_b200_bench --kernel K --matrix M.bin [--lib L.so] [--config JSON]"
                     " [--iters N] [--warmup N] [--K 32] [--tile T --tpr P --unroll U --vec V --block B"
                     " --split rowwise|merge|stream]\n";
        return 2;
    }
    if (args.lib.empty()) args.lib = default_lib(argv[0]);
    const Matrix m = load_tgm1(args.matrix);
    const int64_t M = m.rows, N = m.cols, nnz = m.nnz, K = args.K;

    void* handle = dlopen(args.lib.c_str(), RTLD_NOW);
    if (!handle) die(3, std::string("dlopen failed: ") + dlerror());
    const std::string sym = "launch_" + args.kernel;
    void* fn = dlsym(handle, sym.c_str());
    if (!fn) die(3, "symbol " + sym + " not found in " + args.lib);

    // schedule (only libraries with the native API have one)
    using SetSched = int (*)(const tg_sched*);
    using DefSched = void (*)(tg_sched*);
    using LastStatus = int (*)();
    using LastError = const char* (*)();
    auto set_sched = reinterpret_cast<SetSched>(dlsym(handle, "tg_set_schedule"));
    auto def_sched = reinterpret_cast<DefSched>(dlsym(handle, "tg_default_schedule"));
    auto last_status = reinterpret_cast<LastStatus>(dlsym(handle, "tg_last_status"));
    auto last_error = reinterpret_cast<LastError>(dlsym(handle, "tg_last_error_string"));
    std::string sched_json = "null";
    if (set_sched && def_sched) {
        tg_sched s;
        def_sched(&s);
        if (args.tile) s.tile = args.tile;
        if (args.tpr) s.threads_per_row = args.tpr;
        if (args.unroll) s.unroll = args.unroll;
        if (args.vec) s.vector_width = args.vec;
        if (args.block) s.block_size = args.block;
        if (args.split == "rowwise") s.split = TG_SPLIT_ROWWISE;
        else if (args.split == "merge") s.split = TG_SPLIT_MERGE;
        else if (args.split == "stream") s.split = TG_SPLIT_STREAM;
        else if (!args.split.empty()) die(2, "--split must be rowwise, merge or stream");
        if (set_sched(&s) != TG_OK) die(2, std::string("schedule rejected: ") + (last_error ? last_error() : ""));
        std::ostringstream o;
        o << "{\"tile\":" << s.tile << ",\"threads_per_row\":" << s.threads_per_row << ",\"unroll\":" << s.unroll
          << ",\"vector_width\":" << s.vector_width << ",\"block_size\":" << s.block_size << ",\"split\":" << s.split
          << "}";
        sched_json = o.str();
    }

    // host inputs: the reference harness's deterministic patterns (cpp/src/harness.cpp:144-151)
    std::vector<double> x(N), w(M), B((size_t)N * K), U((size_t)M * K), V((size_t)N * K);
    for (size_t i = 0; i < x.size(); ++i) x[i] = 0.5 + 0.001 * static_cast<double>(i % 97);
    for (size_t i = 0; i < w.size(); ++i) w[i] = -0.25 + 0.002 * static_cast<double>(i % 53);
    for (size_t i = 0; i < B.size(); ++i) B[i] = 0.1 * (static_cast<double>(i % 31) - 15.0);
    for (size_t i = 0; i < U.size(); ++i) U[i] = 0.05 * (static_cast<double>(i % 23) - 11.0);
    for (size_t i = 0; i < V.size(); ++i) V[i] = -0.03 * (static_cast<double>(i % 19) - 9.0);
    const double alpha = 0.7, beta = -1.3;

    // host evaluation of the formula (the check) and the reference's flop/byte model
    std::vector<double> ref;
    double flops = 0.0, bytes = 0.0;
    size_t out_n = 0;
    if (args.kernel == "spmv" || args.kernel == "fused_spmv_axpy") {
        ref.assign(M, 0.0);
        for (int64_t i = 0; i < M; ++i) {
            double acc = 0.0;
            for (int64_t p = m.indptr[i]; p < m.indptr[i + 1]; ++p) acc += m.data[p] * x[m.indices[p]];
            ref[i] = args.kernel == "spmv" ? acc : alpha * acc + beta * w[i];
        }
        flops = 2.0 * nnz;
        bytes = nnz * 16.0 + (M + 1) * 8.0 + nnz * 8.0 + M * 8.0 * (args.kernel == "spmv" ? 1 : 2);
        out_n = M;
    } else if (args.kernel == "spmm") {
        ref.assign((size_t)M * K, 0.0);
        for (int64_t i = 0; i < M; ++i)
            for (int64_t p = m.indptr[i]; p < m.indptr[i + 1]; ++p)
                for (int64_t k = 0; k < K; ++k) ref[(size_t)i * K + k] += m.data[p] * B[(size_t)m.indices[p] * K + k];
        flops = 2.0 * nnz * K;
        bytes = nnz * 16.0 + (M + 1) * 8.0 + nnz * K * 8.0 + M * K * 8.0;
        out_n = (size_t)M * K;
    } else if (args.kernel == "sddmm") {
        ref.assign(nnz, 0.0);
        for (int64_t i = 0; i < M; ++i)
            for (int64_t p = m.indptr[i]; p < m.indptr[i + 1]; ++p) {
                double d = 0.0;
                for (int64_t k = 0; k < K; ++k) d += U[(size_t)i * K + k] * V[(size_t)m.indices[p] * K + k];
                ref[p] = m.data[p] * d;
            }
        flops = 2.0 * nnz * K;
        bytes = nnz * 16.0 + (M + 1) * 8.0 + 2.0 * nnz * K * 8.0 + nnz * 8.0;
        out_n = nnz;
    } else if (args.kernel == "axpy") {
        ref.assign(M, 0.0);
        for (int64_t i = 0; i < M; ++i) ref[i] = alpha * x[i] + beta * w[i];
        flops = 2.0 * M;
        bytes = 3.0 * M * 8.0;
        out_n = M;
    } else {
        die(2, "unknown kernel " + args.kernel);
    }

    // device operands (copied once, outside the timed region)
    int64_t* d_ip = to_device(m.indptr);
    int64_t* d_ix = to_device(m.indices);
    double* d_dv = to_device(m.data);
    double* d_x = to_device(x);
    double* d_w = to_device(w);
    double* d_B = args.kernel == "spmm" ? to_device(B) : nullptr;
    double* d_U = args.kernel == "sddmm" ? to_device(U) : nullptr;
    double* d_V = args.kernel == "sddmm" ? to_device(V) : nullptr;
    double* d_out = nullptr;
    check(cudaMalloc(&d_out, std::max<size_t>(out_n, 1) * sizeof(double)), "cudaMalloc");

    auto run_once = [&]() {
        if (args.kernel == "spmv") {
            using F = void (*)(const int64_t*, const int64_t*, const double*, const double*, double*, int64_t, int64_t,
                               int64_t);
            reinterpret_cast<F>(fn)(d_ip, d_ix, d_dv, d_x, d_out, M, N, nnz);
        } else if (args.kernel == "spmm") {
            using F = void (*)(const int64_t*, const int64_t*, const double*, const double*, double*, int64_t, int64_t,
                               int64_t, int64_t);
            // the reference ABI accumulates into C; the caller zeroes it (tilegen/verify.py:437)
            check(cudaMemset(d_out, 0, out_n * sizeof(double)), "cudaMemset");
            reinterpret_cast<F>(fn)(d_ip, d_ix, d_dv, d_B, d_out, M, N, K, nnz);
        } else if (args.kernel == "sddmm") {
            using F = void (*)(const int64_t*, const int64_t*, const double*, const double*, const double*, double*,
                               int64_t, int64_t, int64_t, int64_t);
            reinterpret_cast<F>(fn)(d_ip, d_ix, d_dv, d_U, d_V, d_out, M, N, K, nnz);
        } else if (args.kernel == "fused_spmv_axpy") {
            using F = void (*)(const int64_t*, const int64_t*, const double*, const double*, const double*, double*,
                               double, double, int64_t, int64_t, int64_t);
            reinterpret_cast<F>(fn)(d_ip, d_ix, d_dv, d_x, d_w, d_out, alpha, beta, M, N, nnz);
        } else {
            using F = void (*)(const double*, const double*, double*, double, double, int64_t);
            reinterpret_cast<F>(fn)(d_x, d_w, d_out, alpha, beta, M);
        }
        if (last_status && last_status() != TG_OK)
            die(5, std::string(sym) + " failed: " + (last_error ? last_error() : "unknown error"));
    };

    for (int i = 0; i < args.warmup; ++i) run_once();
    check(cudaDeviceSynchronize(), "warm-up");
    cudaEvent_t e0, e1;
    check(cudaEventCreate(&e0), "cudaEventCreate");
    check(cudaEventCreate(&e1), "cudaEventCreate");
    std::vector<double> times;
    for (int i = 0; i < args.iters; ++i) {
        check(cudaEventRecord(e0), "cudaEventRecord");
        run_once();
        check(cudaEventRecord(e1), "cudaEventRecord");
        check(cudaEventSynchronize(e1), "cudaEventSynchronize");
        float ms = 0.f;
        check(cudaEventElapsedTime(&ms, e0, e1), "cudaEventElapsedTime");
        times.push_back(ms);
    }
    double sum = 0.0, mn = times[0];
    for (double t : times) {
        sum += t;
        mn = std::min(mn, t);
    }
    const double mean = sum / times.size();

    std::vector<double> out(out_n);
    if (out_n) check(cudaMemcpy(out.data(), d_out, out_n * sizeof(double), cudaMemcpyDeviceToHost), "D2H");
    double max_abs = 0.0, max_rel = 0.0;
    for (size_t i = 0; i < out_n; ++i) {
        const double d = std::fabs(out[i] - ref[i]);
        max_abs = std::max(max_abs, d);
        max_rel = std::max(max_rel, d / std::max(std::fabs(ref[i]), 1e-300));
    }
    const double gflops = mn > 0.0 ? flops / (mn * 1e6) : 0.0;
    const double bw = mn > 0.0 ? bytes / (mn * 1e6) : 0.0;

    cudaDeviceProp prop{};
    int dev = 0;
    check(cudaGetDevice(&dev), "cudaGetDevice");
    check(cudaGetDeviceProperties(&prop, dev), "cudaGetDeviceProperties");
    std::ostringstream js;
    js << "{\"kernel\":\"" << json_escape(args.kernel) << "\",\"config\":" << args.config
       << ",\"backend\":\"b200\",\"schedule\":" << sched_json << ",\"device\":\"" << json_escape(prop.name)
       << "\",\"lib\":\"" << json_escape(args.lib) << "\",\"matrix\":\"" << json_escape(args.matrix)
       << "\",\"rows\":" << M << ",\"cols\":" << N << ",\"nnz\":" << nnz << ",\"K\":" << K << ",\"ms_mean\":" << mean
       << ",\"ms_min\":" << mn << ",\"gflops\":" << gflops << ",\"bandwidth_gbs\":" << bw
       << ",\"max_abs_err\":" << max_abs << ",\"max_rel_err\":" << max_rel << "}";
    std::cout << js.str() << std::endl;

    for (void* p : {(void*)d_ip, (void*)d_ix, (void*)d_dv, (void*)d_x, (void*)d_w, (void*)d_B, (void*)d_U, (void*)d_V,
                    (void*)d_out})
        if (p) cudaFree(p);
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    dlclose(handle);
    return 0;
}
