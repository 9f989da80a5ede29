"""Benchmark of the b200 sparse hot path (one JSON line on rank 0).

Workload (the configuration the 1/2/4/8-GPU metric is quoted
on, which fits one B200): C4 -- an 8,000,000 x 8,000,000 CSR matrix with 32 distinct
uniformly drawn columns per row (256M nonzeros, int64 indices, fp64 values U(-1,1)),
row-sharded nnz-balanced over the N GPUs, and 20 power iterations x <- A x / ||A x||
from a seeded U(-1,1) x0.  One STEP is one such 20-iteration solve (set x0, 20 fused
SpMV+norm kernels with the shard exchange between them, finalise).  Strong scaling:
the matrix is the same at every N.

Metric: effective HBM GB/s = compulsory SpMV bytes (8(M+1) + 16 nnz + 8 N + 8 M for the
whole matrix) x 20 iterations / step time, whole job, max over ranks.  `value` has A and
x0 resident in HBM; `e2e` repeats the step through the public API from pinned host
buffers (H2D of the shard, column renumbering, 20 iterations, D2H of x and lambda).
The inputs (4.29 GB) exceed the 126 MB L2, so no flush is needed between steps.  On one
GPU the line also carries `cusparse` (cuSPARSE SpMV on the same arrays).

The same line carries `workloads`: the other BASELINE configurations (C1 uniform, C2
banded, C3 power-law SpMV; C5 SpMM K=128 and SDDMM K=64), each row-sharded over the same
ranks and timed the same way (L2 flushed before each call where the problem fits in L2),
with ms, effective GB/s, roofline fraction, cuSPARSE and the reference's CPU kernel
beside it.  `--workload c1|c2|c3|c5-spmm|c5-sddmm` prints one of them as its own line.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
"""

from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

REPO = os.path.dirname(os.path.abspath(__file__))
if REPO not in sys.path:
    sys.path.insert(0, REPO)

C4_N = 8_000_000
C4_PER_ROW = 32
C4_SEED = 4
X0_SEED = 7
ITERS = 20
FALLBACK_HBM_GBS = 6650.0

WORKLOADS = ("c4", "c1", "c2", "c3", "c5-spmm", "c5-sddmm", "c5-spmm-rcm", "blocked-spmm")
# Default schedule per workload: the fastest measured in the schedule sweeps on a B200.
SCHEDULES = {
    "c4": {"split": "rowwise", "tpr": 4, "unroll": 1, "vec": 4, "block": 256},
    "c1": {"split": "rowwise", "tpr": 4, "unroll": 2, "vec": 2, "block": 128},
    "c2": {"split": "merge", "tpr": 8, "unroll": 2, "vec": 2, "block": 256},
    "c3": {"split": "merge", "tpr": 8, "unroll": 2, "vec": 2, "block": 256},
    "c5-spmm": {"split": "merge", "tpr": 32, "unroll": 4, "vec": 4, "block": 128},
    "c5-sddmm": {"split": "merge", "tpr": 8, "unroll": 1, "vec": 4, "block": 128},
    "c5-spmm-rcm": {"split": "merge", "tpr": 32, "unroll": 4, "vec": 4, "block": 128},
    "blocked-spmm": {"split": "block", "tpr": 32, "unroll": 4, "vec": 4, "block": 256},
}
# C4 on N > 1 GPUs with the fused exchange: int64 indices, TPR4 U2 V2.  Measured at N=2
# against the one-GPU default (int32, TPR4 U1 V4): 5899 vs 5424 GB/s; the faster
# compute-only step (0.593 vs 0.625 ms) loses more to its exposed exchange (0.198 vs
# 0.102 ms per iteration).
C4_FUSED_SCHEDULE = {"split": "rowwise", "tpr": 4, "unroll": 2, "vec": 2, "block": 256}


def parse():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--rows", type=int, default=C4_N, help="matrix size (default: the C4 config)")
    ap.add_argument("--iters", type=int, default=ITERS)
    ap.add_argument("--e2e-steps", type=int, default=3)
    ap.add_argument("--workload", choices=WORKLOADS, default="c4",
                    help="c4: the power-iteration headline (default); c1/c2/c3: one SpMV per step; "
                         "c5-spmm / c5-sddmm: one SpMM (K=128) / SDDMM (K=64) per step, fp32")
    ap.add_argument("--split", choices=["stream", "rowwise", "merge", "block"], default=None)
    ap.add_argument("--exchange", choices=["p2p", "ce", "nccl"], default="p2p",
                    help="N>1: fused SpMV + peer-memory push (p2p), plain step + one copy-engine copy per peer "
                         "(ce), or NCCL all-gather")
    ap.add_argument("--ce-chunks", type=int, default=4, help="--exchange ce: row chunks per step (1-16)")
    ap.add_argument("--tpr", type=int, default=None)
    ap.add_argument("--unroll", type=int, default=None)
    ap.add_argument("--vec", type=int, default=None)
    ap.add_argument("--block", type=int, default=None)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-cusparse", action="store_true")
    ap.add_argument("--index-bits", type=int, choices=[32, 64], default=None,
                    help="c4: width of the renumbered column indices the power steps stream (32: 12 bytes "
                         "per nonzero, 64: 16); default 32 on one GPU, 64 with the fused exchange")
    ap.add_argument("--no-workloads", action="store_true",
                    help="c4: skip the C1-C3 / C5 measurements that the default line carries in `workloads`")
    args = ap.parse_args()
    d = SCHEDULES[args.workload]
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if args.workload == "c4" and world > 1 and args.exchange == "p2p":
        d = C4_FUSED_SCHEDULE
    for k in ("split", "tpr", "unroll", "vec", "block"):
        if getattr(args, k) is None:
            setattr(args, k, d[k])
    if args.index_bits is None:
        args.index_bits = 64 if (args.workload == "c4" and world > 1 and args.exchange == "p2p") else 32
    return args


def spmv_bytes(rows: int, cols: int, nnz: int) -> int:
    """Compulsory bytes of one CSR SpMV: indptr + indices + values + x + y."""
    return 8 * (rows + 1) + 16 * nnz + 8 * cols + 8 * rows


def measured_peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as fh:
            d = json.load(fh)
        return float(d["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


def traffic_record(workload: str, kernel: str):
    """dram bytes per launch from the committed ncu summary (profiles/traffic.json)."""
    path = os.path.join(REPO, "profiles", "traffic.json")
    if not os.path.exists(path):
        return None
    with open(path) as fh:
        d = json.load(fh)
    rec = d.get(workload, {}).get(kernel)
    return rec


class ClockSampler:
    """nvidia-smi clocks/throttle sampling during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.first = ""

    def start(self):
        """Start sampling and wait (up to 5 s) for the first sample, so that a timed region
        shorter than the sampling period still has the sample taken as it begins."""
        import select

        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.idx), "--query-gpu=" + self.FIELDS,
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        ready, _, _ = select.select([self.proc.stdout], [], [], 5.0)
        if ready:
            self.first = self.proc.stdout.readline()

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        out = self.first + out
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.splitlines():
            f = [c.strip() for c in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax.append(float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(smax), "reasons": sorted(reasons),
                "samples": len(sm)}


# ----------------------------------------------------------------------------- CPU legs
def cpu_reference_spmv(A, x_len: int):
    """The reference's own OpenMP SpMV (oracle/_ref, rebuilt with -march=native when a
    compiler exists) or, failing that, the oracle's OpenMP port.  Returns
    (callable(x, y), kind, description, threads)."""
    from oracle import build as ob
    from oracle import oracle as O

    threads = os.cpu_count() or 1
    os.environ.setdefault("OMP_NUM_THREADS", str(threads))
    libs = None
    native_dir = os.path.join("/tmp", "tilegen_ref_native")
    if os.path.exists(ob.GEN_DIR):
        libs = ob.rebuild_ref_native(native_dir)
        march = "native"
        if not libs:
            libs = O.ref_omp_libs()
            march = "x86-64-v3"
    if libs:
        M, N, nnz = A.rows, A.cols, A.nnz
        ip, ix, d = A.indptr, A.indices, A.data
        best = None
        for cfg in ("T32U1", "T64U2", "T128U4"):  # small CPU autotune, budget 3
            stem = "ref_omp_spmv_f64_%s" % cfg
            if stem not in libs:
                continue
            k = O.RefOmpKernel(libs[stem], "spmv")
            y = np.empty(M)
            xx = np.ones(N)
            k(ip, ix, d, xx, y, M, N, nnz)
            t0 = time.perf_counter()
            k(ip, ix, d, xx, y, M, N, nnz)
            dt = time.perf_counter() - t0
            if best is None or dt < best[0]:
                best = (dt, cfg, k)
        if best is not None:
            k = best[2]
            return ((lambda x, y: k(ip, ix, d, x, y, M, N, nnz)), "reference",
                    "reference OpenMP launch_spmv (tilegen codegen cpu backend, %s, -O3 -march=%s -fopenmp)"
                    % (best[1], march), threads)
    return ((lambda x, y: O.spmv_omp(A, x, out=y)), "port", "oracle OpenMP port of cpp/src/ref.cpp:6-15", threads)


def cpu_power_sample(A, x0, iters: int, spmv):
    """`iters` power iterations on the host; returns seconds."""
    x = x0.copy()
    y = np.empty(A.rows)
    t0 = time.perf_counter()
    for _ in range(iters):
        spmv(x, y)
        nrm = float(np.sqrt(np.dot(y, y)))
        np.multiply(y, 1.0 / nrm, out=x)
    return time.perf_counter() - t0


def run_reference(args, rank: int, world: int):
    """--impl reference: the reference's CPU implementation of the path, rank 0 only."""
    if rank != 0:
        return 0
    from tilegen_b200 import matrices as Mx

    n = args.rows
    A = Mx.c4_rows(0, n, n=n, per_row=C4_PER_ROW, seed=C4_SEED)
    x0 = np.random.default_rng([X0_SEED, 0]).uniform(-1.0, 1.0, size=n)
    spmv, kind, desc, threads = cpu_reference_spmv(A, n)
    iters_per_step = 2
    for _ in range(args.warmup):
        cpu_power_sample(A, x0, 1, spmv)
    times = [cpu_power_sample(A, x0, iters_per_step, spmv) for _ in range(args.steps)]
    bytes_iter = spmv_bytes(n, n, A.nnz)
    sec = float(np.mean(times))
    gbs = bytes_iter * iters_per_step / sec / 1e9
    sample = "%d of the %d power iterations per step on the full %dx%d matrix (%d nnz)" % (
        iters_per_step, ITERS, n, n, A.nnz)
    line = {
        "impl": "reference",
        "metric": "effective_hbm_gbs_power_iteration_spmv",
        "value": round(gbs, 3),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(sec * 1e3, 3),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "f64",
        "data": "synthetic (seeded C4 generator)",
        "config": workload_config(n, world),
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": kind,
                         "sample": sample, "impl": desc},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def workload_config(n: int, world: int, exchange: str = "p2p"):
    return {"workload": "C4 power iteration: %dx%d CSR, %d distinct cols/row, fp64, %d iterations/step"
                        % (n, n, C4_PER_ROW, ITERS),
            "rows": n, "nnz": n * C4_PER_ROW, "iterations_per_step": ITERS,
            "parallelism": ("single GPU, no exchange" if world == 1 else
                            "row-sharded x%d, x replicated (%s)" % (
                                world, {"p2p": "fused SpMV + peer-memory push of shards",
                                        "ce": "SpMV, then one copy-engine copy of the shard per peer",
                                        "nccl": "in-place NCCL all-gather of shards"}[exchange])),
            "l2": "inputs (%.2f GB) larger than L2 (126 MB): no flush" % (spmv_bytes(n, n, n * C4_PER_ROW) / 1e9)}


# ----------------------------------------------------------------------------- C1-C3, C5
K_DENSE = {"c5-spmm": 128, "c5-sddmm": 64, "c5-spmm-rcm": 128, "blocked-spmm": 128}
SPMM_WORKLOADS = ("c5-spmm", "c5-spmm-rcm", "blocked-spmm")
FP32_WORKLOADS = ("c5-spmm", "c5-sddmm", "c5-spmm-rcm", "blocked-spmm")
INPUT_SEED = 11


def matrix_kernel(workload: str) -> str:
    return {"c5-sddmm": "sddmm"}.get(workload, "spmm" if workload in SPMM_WORKLOADS else "spmv")


def matrix_bytes(workload: str, A) -> int:
    """Compulsory bytes of one call on the whole matrix: indptr + indices + values + dense
    inputs + outputs, each once (8-byte indices; fp64 for SpMV, fp32 for C5)."""
    M, N, nnz = A.rows, A.cols, A.nnz
    if workload in FP32_WORKLOADS:
        K = K_DENSE[workload]
        base = 8 * (M + 1) + 12 * nnz
        if workload in SPMM_WORKLOADS:
            return base + 4 * N * K + 4 * M * K
        return base + 4 * M * K + 4 * N * K + 4 * nnz
    return spmv_bytes(M, N, nnz)


def matrix_flops(workload: str, A) -> float:
    if workload in FP32_WORKLOADS:
        return 2.0 * A.nnz * K_DENSE[workload] + (A.nnz if workload == "c5-sddmm" else 0)
    return 2.0 * A.nnz


def matrix_inputs(workload: str, A):
    """Seeded U(-1,1) dense operands: x (fp64) for SpMV, B (N x 128) or U (M x 64),
    V (N x 64) in fp32 for C5."""
    rng = np.random.default_rng([INPUT_SEED, 0])
    if workload in SPMM_WORKLOADS:
        return {"B": rng.uniform(-1.0, 1.0, size=(A.cols, 128)).astype(np.float32)}
    if workload == "c5-sddmm":
        U = rng.uniform(-1.0, 1.0, size=(A.rows, 64)).astype(np.float32)
        V = rng.uniform(-1.0, 1.0, size=(A.cols, 64)).astype(np.float32)
        return {"U": U, "V": V}
    return {"x": rng.uniform(-1.0, 1.0, size=A.cols)}


def row_shard(A, r0: int, r1: int):
    from tilegen_b200.matrices import CSR

    p0, p1 = int(A.indptr[r0]), int(A.indptr[r1])
    return CSR(A.indptr[r0:r1 + 1] - p0, A.indices[p0:p1], A.data[p0:p1], (r1 - r0, A.cols),
               "%s[%d:%d]" % (A.name, r0, r1))


def matrix_config(workload: str, A, world: int, flush: bool):
    desc = {"c1": "C1 uniform_random 100000^2, 16 distinct cols/row, fp64 SpMV",
            "c2": "C2 banded 200000^2, offsets -3..3 clipped, fp64 SpMV",
            "c3": "C3 power_law 100000^2, Zipf(2) rows scaled to mean 8, fp64 SpMV",
            "c5-spmm": "C5 SpMM: power_law 1000000^2 (Zipf(2), mean 16) x dense 1000000x128, fp32",
            "c5-sddmm": "C5 SDDMM: power_law 1000000^2 (Zipf(2), mean 16) pattern, U,V 1000000x64, fp32",
            "c5-spmm-rcm": "C5 SpMM after reverse Cuthill-McKee reordering (labelled configuration: A' = P A P^T, "
                           "B' = P B, C' = P C; changes the input order)",
            "blocked-spmm": "SpMM K=128 fp32 on the reference corpus's blocked class (100000^2, dense 8x8 blocks, "
                            "2 per block row; labelled configuration for block-structured matrices)"}[workload]
    return {"workload": desc, "rows": A.rows, "cols": A.cols, "nnz": A.nnz,
            "max_row_nnz": int(np.diff(A.indptr).max()) if A.rows else 0,
            "parallelism": "single GPU" if world == 1 else
            "row-sharded x%d (nnz-balanced), dense operands replicated, no communication" % world,
            "l2": ("host run" if flush is None else
                   "L2 flushed (256 MB write) before every step, outside the step's events" if flush else
                   "inputs larger than L2 (126 MB): no flush")}


def cpu_reference_kernel(kernel: str, dtype: str):
    """The reference's OpenMP launch_<kernel> (best of its three CPU configs on one call),
    or None when the reference build is absent.  Returns (make_call, description)."""
    from oracle import build as ob
    from oracle import oracle as O

    threads = os.cpu_count() or 1
    os.environ.setdefault("OMP_NUM_THREADS", str(threads))
    if not os.path.exists(ob.GEN_DIR):
        return None
    libs = ob.rebuild_ref_native(os.path.join("/tmp", "tilegen_ref_native"))
    march = "native"
    if not libs:
        libs, march = O.ref_omp_libs(), "x86-64-v3"
    cands = [(cfg, libs["ref_omp_%s_%s_%s" % (kernel, dtype, cfg)]) for cfg in ("T32U1", "T64U2", "T128U4")
             if "ref_omp_%s_%s_%s" % (kernel, dtype, cfg) in libs]
    if not cands:
        return None
    return [(cfg, O.RefOmpKernel(path, kernel)) for cfg, path in cands], march, threads


def cpu_matrix_caller(workload: str, A, inputs):
    """A zero-argument call of the reference's OpenMP kernel on the whole matrix (its best
    of three CPU configs, chosen once), else of the oracle's OpenMP SpMV port.  Returns
    (call or None, kind, description, threads)."""
    from oracle import oracle as O

    kernel = matrix_kernel(workload)
    dtype = "f32" if workload in FP32_WORKLOADS else "f64"
    M, N, nnz = A.rows, A.cols, A.nnz
    ip, ix = A.indptr, A.indices
    d = A.data.astype(np.float32) if dtype == "f32" else A.data
    if kernel == "spmv":
        out = np.empty(M)
        args = (ip, ix, d, inputs["x"], out, M, N, nnz)
    elif kernel == "spmm":
        out = np.zeros((M, 128), dtype=np.float32)
        args = (ip, ix, d, inputs["B"], out, M, N, 128, nnz)
    else:
        out = np.zeros(nnz, dtype=np.float32)
        args = (ip, ix, d, inputs["U"], inputs["V"], out, M, N, 64, nnz)
    threads = os.cpu_count() or 1
    ref = cpu_reference_kernel(kernel, dtype)
    if ref is not None:
        cands, march, threads = ref
        best = None
        for cfg, k in cands:
            k(*args)
            t0 = time.perf_counter()
            k(*args)
            dt = time.perf_counter() - t0
            if best is None or dt < best[0]:
                best = (dt, cfg, k)
        _, cfg, k = best
        return ((lambda: k(*args)), "reference",
                "reference OpenMP launch_%s (tilegen codegen cpu backend, %s, %s, -O3 -march=%s -fopenmp)"
                % (kernel, dtype, cfg, march), threads)
    if kernel != "spmv":
        return None, "port", "no reference OpenMP build of launch_%s on this host" % kernel, threads
    x = inputs["x"]
    return (lambda: O.spmv_omp(A, x, out=out)), "port", "oracle OpenMP port of cpp/src/ref.cpp:6-15", threads


def cpu_matrix_sample(workload: str, A, inputs, reps: int):
    """(seconds per whole-matrix call, kind, description, threads) over `reps` calls."""
    call, kind, desc, threads = cpu_matrix_caller(workload, A, inputs)
    if call is None:
        return None, kind, desc, threads
    t0 = time.perf_counter()
    for _ in range(reps):
        call()
    return (time.perf_counter() - t0) / reps, kind, desc, threads


def run_matrix_reference(args, rank: int, world: int):
    """--impl reference for C1-C3/C5: the reference's OpenMP kernel on the host cores, one
    whole-matrix call per step, rank 0 only."""
    if rank != 0:
        return 0
    from tilegen_b200 import matrices as Mx

    A = (Mx.make_matrix("blocked") if args.workload == "blocked-spmm" else
         Mx.baseline_matrix("c5" if args.workload.startswith("c5") else args.workload))
    inputs = matrix_inputs(args.workload, A)
    call, kind, desc, threads = cpu_matrix_caller(args.workload, A, inputs)
    if call is None:
        print(json.dumps({"impl": "reference", "unavailable": desc}), flush=True)
        return 0
    for _ in range(args.warmup):
        call()
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        call()
        times.append(time.perf_counter() - t0)
    sec = float(np.mean(times))
    gbs = matrix_bytes(args.workload, A) / sec / 1e9
    line = {"impl": "reference", "metric": "effective_hbm_gbs_" + matrix_kernel(args.workload), "value": round(gbs, 3),
            "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(sec * 1e3, 4), "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "f32" if args.workload in FP32_WORKLOADS else "f64", "data": "synthetic (seeded generators)",
            "config": matrix_config(args.workload, A, world, None),
            "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": kind,
                             "sample": "one whole-matrix call per step", "impl": desc},
            "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def make_sched(split: str, tpr: int, unroll: int, vec: int, block: int):
    from tilegen_b200 import lib

    sch = lib.default_schedule()
    sch.threads_per_row, sch.unroll, sch.vector_width, sch.block_size, sch.tile = tpr, unroll, vec, block, 32
    sch.split = {"rowwise": lib.TG_SPLIT_ROWWISE, "merge": lib.TG_SPLIT_MERGE, "stream": lib.TG_SPLIT_STREAM,
                 "block": lib.TG_SPLIT_BLOCK}[split]
    lib.validate_schedule(sch)
    return sch


def measure_matrix(wl: str, sched: dict, steps: int, warmup: int, rank: int, world: int, dev, barrier,
                   e2e_steps: int, want_cpu: bool, want_cusparse: bool, sample_clocks: bool):
    """One C1-C3 / C5 workload: rank `rank`'s row shard (nnz-balanced, dense operands
    replicated), `steps` timed calls after `warmup`, L2 flushed before each call when the
    problem fits in L2.  Returns the measurement record (times are this rank's; the
    caller takes the max over ranks)."""
    import torch

    from tilegen_b200 import device as D
    from tilegen_b200 import lib, matrices as Mx
    from tilegen_b200.power import nnz_balanced_bounds

    L = lib.load()
    kernel = matrix_kernel(wl)
    c5 = wl in FP32_WORKLOADS
    A = Mx.make_matrix("blocked") if wl == "blocked-spmm" else Mx.baseline_matrix("c5" if wl.startswith("c5") else wl)
    inputs = matrix_inputs(wl, A)
    reorder = None
    if wl.endswith("-rcm"):
        from tilegen_b200 import reorder as Ro

        t0 = time.perf_counter()
        perm = Ro.rcm_order(A)
        t1 = time.perf_counter()
        bw0 = Ro.bandwidth(A)
        A = Ro.permute(A, perm)
        inputs = {k: Ro.permute_rows(v, perm) for k, v in inputs.items()}
        reorder = {"order": "reverse Cuthill-McKee (tg_rcm_order, host)", "order_s": round(t1 - t0, 3),
                   "permute_s": round(time.perf_counter() - t1, 3), "bandwidth_before": bw0,
                   "bandwidth_after": Ro.bandwidth(A)}
    bounds = nnz_balanced_bounds(np.diff(A.indptr), world)
    r0, r1 = int(bounds[rank]), int(bounds[rank + 1])
    S = row_shard(A, r0, r1)
    dt = torch.float32 if c5 else torch.float64
    Ad = D.DeviceCSR.from_host(S, dev, dt)
    sch = make_sched(sched["split"], sched["tpr"], sched["unroll"], sched["vec"], sched["block"])

    # pinned host inputs (e2e) and their device copies
    h_in = {k: torch.from_numpy(np.ascontiguousarray(v[r0:r1] if k == "U" else v)).pin_memory()
            for k, v in inputs.items()}
    d_in = {k: v.to(dev, dtype=dt) for k, v in h_in.items()}
    plan = None
    if kernel == "spmv":
        out = torch.empty(S.rows, dtype=dt, device=dev)
        if sched["split"] in ("merge", "stream"):
            # the partition of the matrix (the plan) is computed by the first call into a
            # workspace of this workload's own and reused by every later call
            ws = torch.zeros(int(L.tg_spmv_workspace_bytes(S.rows, S.nnz, ctypes.byref(sch))), dtype=torch.uint8,
                             device=dev)
            torch.cuda.synchronize(dev)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            D.spmv(Ad, d_in["x"], out, sched=sch, workspace=ws)  # planning call
            e1.record()
            torch.cuda.synchronize(dev)
            plan = {"first_call_ms": round(e0.elapsed_time(e1), 5),
                    "note": "partition computed by the first call, reused by every timed call (TG_FLAG_REUSE_PLAN)"}
            sch_r = make_sched(sched["split"], sched["tpr"], sched["unroll"], sched["vec"], sched["block"])
            sch_r.flags |= lib.TG_FLAG_REUSE_PLAN
            step = lambda: D.spmv(Ad, d_in["x"], out, sched=sch_r, workspace=ws)  # noqa: E731
        else:
            step = lambda: D.spmv(Ad, d_in["x"], out, sched=sch)  # noqa: E731
    elif kernel == "spmm":
        out = torch.empty((S.rows, 128), dtype=dt, device=dev)
        if sched["split"] == "block":
            # the row-group flags (the plan) are computed by the first call and reused
            ws = torch.zeros(max(1, int(L.tg_spmm_workspace_bytes(S.rows, S.nnz, 128, ctypes.byref(sch)))),
                             dtype=torch.uint8, device=dev)
            torch.cuda.synchronize(dev)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            D.spmm(Ad, d_in["B"], out, sched=sch, workspace=ws)  # planning call
            e1.record()
            torch.cuda.synchronize(dev)
            plan = {"first_call_ms": round(e0.elapsed_time(e1), 5),
                    "note": "row-group flags computed by the first call, reused by every timed call "
                            "(TG_FLAG_REUSE_PLAN)"}
            sch_r = make_sched(sched["split"], sched["tpr"], sched["unroll"], sched["vec"], sched["block"])
            sch_r.flags |= lib.TG_FLAG_REUSE_PLAN
            step = lambda: D.spmm(Ad, d_in["B"], out, sched=sch_r, workspace=ws)  # noqa: E731
        else:
            step = lambda: D.spmm(Ad, d_in["B"], out, sched=sch)  # noqa: E731
    else:
        out = torch.empty(S.nnz, dtype=dt, device=dev)
        step = lambda: D.sddmm(Ad, d_in["U"], d_in["V"], out, sched=sch)  # noqa: E731
    h_out = torch.empty(out.shape, dtype=dt).pin_memory()
    flush_needed = matrix_bytes(wl, A) < (256 << 20)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev) if flush_needed else None
    stream = torch.cuda.current_stream(dev)

    for _ in range(warmup):
        step()
    barrier()
    sampler = ClockSampler(dev.index) if sample_clocks else None
    if sampler:
        sampler.start()
    barrier()
    n0 = L.tg_launch_count()
    evs = []
    wall0 = time.perf_counter()
    for _ in range(steps):
        if flush is not None:
            flush.zero_()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        step()
        e1.record(stream)
        evs.append((e0, e1))
    barrier()
    wall = time.perf_counter() - wall0
    launches = L.tg_launch_count() - n0
    clocks = sampler.stop() if sampler else None
    ms_local = float(np.mean([a.elapsed_time(b) for a, b in evs]))

    # problems that fit in L2: also the event pair's own floor after the same flush (an
    # empty one-element op), and the warm per-call time (20 back-to-back calls captured
    # in a CUDA graph, inputs L2-resident), so the cold time can be read against both
    floor = None
    if flush is not None:
        tiny = torch.zeros(1, device=dev)
        fe = []
        for _ in range(max(steps, 5)):
            flush.zero_()
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            tiny.add_(1.0)
            e1.record(stream)
            fe.append((e0, e1))
        torch.cuda.synchronize(dev)
        warm_ms = warm_graph_ms(step, dev)
        floor = {"event_floor_ms": round(float(np.median([a.elapsed_time(b) for a, b in fe])), 5),
                 "warm_ms": round(warm_ms, 5) if warm_ms is not None else None,
                 "what": "event_floor_ms: the same flush then an event pair around a one-element op; "
                         "warm_ms: per call, 20 calls back to back in a CUDA graph, L2-resident"}

    # C5: the dense-row gather floor -- the bench-only probe reads the same B (SpMM) or V
    # (SDDMM) row for every nonzero and nothing else; alternated with the step so both see
    # the same clocks
    row_floor = None
    if c5 and kernel in ("spmm", "sddmm"):
        from tilegen_b200 import bench_probe

        dense = d_in["B"] if kernel == "spmm" else d_in["V"]
        pout = torch.zeros(1, dtype=torch.float64, device=dev)

        def probe():
            bench_probe.row_gather_probe_f32(Ad.indices.data_ptr(), S.nnz, dense.data_ptr(), int(dense.shape[1]),
                                             pout.data_ptr(), stream.cuda_stream)

        for _ in range(3):
            probe()
        pe, se = [], []
        for _ in range(10):
            ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
            ev[0].record(stream)
            probe()
            ev[1].record(stream)
            ev[2].record(stream)
            step()
            ev[3].record(stream)
            pe.append((ev[0], ev[1]))
            se.append((ev[2], ev[3]))
        torch.cuda.synchronize(dev)
        p_ms = float(np.median([a.elapsed_time(b) for a, b in pe]))
        s_ms = float(np.median([a.elapsed_time(b) for a, b in se]))
        row_bytes = int(dense.shape[1]) * dense.element_size()
        row_floor = {"ms": round(p_ms, 5), "step_ms": round(s_ms, 5), "frac": round(p_ms / s_ms, 4),
                     "gathered_gbs": round(S.nnz * row_bytes / (p_ms / 1e3) / 1e9, 1),
                     "what": "tg_row_gather_probe_f32: the %d-byte %s row of every nonzero (same indices, load "
                             "instruction and L2 policy) and nothing else, alternated with the step; frac = "
                             "probe time / step time" % (row_bytes, "B" if kernel == "spmm" else "V")}

    # e2e through the public API: H2D of the step's dense inputs from pinned memory, the
    # call, D2H of the output shard
    e2e = []
    for it in range(e2e_steps + 1 if e2e_steps > 0 else 0):
        barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for k in d_in:
            d_in[k].copy_(h_in[k], non_blocking=True)
        step()
        h_out.copy_(out, non_blocking=True)
        e1.record(stream)
        barrier()
        if it > 0:
            e2e.append(e0.elapsed_time(e1))
    rec = {"wl": wl, "A": A, "S": S, "kernel": kernel, "ms_local": ms_local,
           "e2e_local": float(np.mean(e2e)) if e2e else float("nan"), "launches": int(launches), "clocks": clocks,
           "wall": wall, "flush": flush is not None, "c5": c5, "inputs": inputs, "schedule": dict(sched),
           "h2d": int(sum(v.numel() * v.element_size() for v in h_in.values())),
           "d2h": int(h_out.numel() * h_out.element_size()), "plan": plan, "floor": floor, "reorder": reorder,
           "row_floor": row_floor}
    if want_cusparse:
        rec["cusparse"] = cusparse_compare(wl, Ad, d_in, flush, steps, matrix_bytes(wl, A))
    if want_cpu:
        reps = 3 if c5 else 20
        sec, kind, desc, threads = cpu_matrix_sample(wl, A, inputs, reps)
        if sec is not None:
            rec["cpu_baseline"] = {"value": round(matrix_bytes(wl, A) / sec / 1e9, 3), "unit": "GB/s",
                                   "cores": threads, "kind": kind,
                                   "sample": "%d whole-matrix calls on the host cores" % reps, "impl": desc}
    return rec


def warm_graph_ms(step, dev, calls: int = 20, replays: int = 5):
    """Per-call time of `calls` back-to-back calls captured in one CUDA graph (inputs
    L2-resident), or None when the call cannot be captured."""
    import torch

    try:
        g = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            step()
        torch.cuda.synchronize(dev)
        with torch.cuda.graph(g, stream=side):
            for _ in range(calls):
                step()
        g.replay()
        torch.cuda.synchronize(dev)
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(replays):
            g.replay()
        b.record()
        torch.cuda.synchronize(dev)
        return a.elapsed_time(b) / (calls * replays)
    except Exception:  # noqa: BLE001 -- a supplementary figure must not fail the bench
        return None


def matrix_kernel_name(kernel: str, split: str) -> str:
    return {"spmv": "spmv_rowwise_kernel" if split == "rowwise" else "spmv_merge_kernel",
            "spmm": "spmm_group_kernel" if split == "block" else "spmm kernel", "sddmm": "sddmm kernel"}[kernel]


def summarise_matrix(rec, ms_step: float, world: int, peak: float):
    """Compact per-workload record for the default run's `workloads` object."""
    wl, A, S = rec["wl"], rec["A"], rec["S"]
    total = matrix_bytes(wl, A)
    local = matrix_bytes(wl, S)
    achieved = local / (rec["ms_local"] / 1e3) / 1e9
    d = {"workload": matrix_config(wl, A, world, rec["flush"])["workload"], "rows": A.rows, "nnz": A.nnz,
         "ms": round(ms_step, 5), "value": round(total / (ms_step / 1e3) / 1e9, 2), "unit": "GB/s",
         "gflops": round(matrix_flops(wl, A) / (ms_step / 1e3) / 1e9, 2),
         "roofline_frac": round(achieved / peak, 4), "algorithmic_bytes": int(total),
         "l2": "flushed before every call" if rec["flush"] else "inputs larger than L2",
         "schedule": rec["schedule"], "gpu_launches": rec["launches"]}
    tr = traffic_record("%s_%d" % (wl, world), matrix_kernel_name(rec["kernel"], rec["schedule"]["split"]))
    d["traffic_bytes"] = tr["dram_bytes_per_launch"] if tr else None
    if rec.get("plan"):
        d["plan"] = rec["plan"]
    if rec.get("floor"):
        d["timing_floor"] = rec["floor"]
    if rec.get("reorder"):
        d["reorder"] = rec["reorder"]
    if rec.get("row_floor"):
        d["row_gather_floor"] = rec["row_floor"]
    if "cusparse" in rec:
        c = rec["cusparse"]
        d["cusparse"] = c
        if "ms_per_step" in c:
            d["vs_cusparse"] = round(c["ms_per_step"] / ms_step, 3)
    if "cpu_baseline" in rec:
        d["cpu_baseline"] = rec["cpu_baseline"]
    return d


def run_matrix_workload(args, rank: int, world: int, local_rank: int):
    """C1-C3 (one SpMV per step) and C5 (one SpMM or SDDMM per step), row-sharded over the
    ranks with the dense operands replicated (strong scaling, no communication)."""
    import torch
    import torch.distributed as dist

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)

    wl = args.workload
    sched = {"split": args.split, "tpr": args.tpr, "unroll": args.unroll, "vec": args.vec, "block": args.block}
    rec = measure_matrix(wl, sched, args.steps, args.warmup, rank, world, dev, barrier, args.e2e_steps,
                         want_cpu=(world == 1 and rank == 0 and not args.no_cpu_baseline),
                         want_cusparse=(world == 1 and not args.no_cusparse), sample_clocks=(rank == 0))
    vals = torch.tensor([rec["ms_local"], rec["e2e_local"]], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(vals, op=dist.ReduceOp.MAX)
    ms_step, e2e_ms = [float(v) for v in vals.cpu()]
    A, S, kernel = rec["A"], rec["S"], rec["kernel"]
    total = matrix_bytes(wl, A)
    gbs = total / (ms_step / 1e3) / 1e9
    if rank == 0:
        peak, peak_kind = measured_peaks()
        local_bytes = matrix_bytes(wl, S)  # this rank's rows, the whole replicated dense input
        achieved = local_bytes / (rec["ms_local"] / 1e3) / 1e9
        kname = matrix_kernel_name(kernel, args.split)
        tr = traffic_record("%s_%d" % (wl, world), kname)
        line = {
            "metric": "effective_hbm_gbs_" + kernel,
            "value": round(gbs, 2),
            "unit": "GB/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms_step, 5),
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": "f32" if rec["c5"] else "f64",
            "data": "synthetic (seeded generators, values U(-1,1))",
            "config": matrix_config(wl, A, world, rec["flush"]),
            "gflops": round(matrix_flops(wl, A) / (ms_step / 1e3) / 1e9, 2),
            "e2e": {"value": round(total / (e2e_ms / 1e3) / 1e9, 2), "unit": "GB/s", "h2d_bytes_per_step": rec["h2d"],
                    "d2h_bytes_per_step": rec["d2h"], "ms_per_step": round(e2e_ms, 4)},
            "gpu_launches": rec["launches"],
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4),
                         "peak_source": (peak_kind + " (MEASURED_PEAKS.json hbm_gbs)") if peak_kind == "measured"
                         else "fallback 6.65 TB/s",
                         "kernel": kname + " (whole call, every launch of the step)",
                         "kernel_ms": round(rec["ms_local"], 5), "algorithmic_bytes_per_launch": int(local_bytes),
                         "traffic": tr["dram_bytes_per_launch"] if tr else None},
            "clocks": rec["clocks"],
            "wall_s_timed": round(rec["wall"], 4),
            "schedule": rec["schedule"],
        }
        if rec.get("plan"):
            line["plan"] = rec["plan"]
        if rec.get("floor"):
            line["timing_floor"] = rec["floor"]
        if rec.get("reorder"):
            line["reorder"] = rec["reorder"]
        if rec.get("row_floor"):
            line["roofline"]["row_gather_floor"] = rec["row_floor"]
        if "cusparse" in rec:
            line["cusparse"] = rec["cusparse"]
        if "cpu_baseline" in rec:
            line["cpu_baseline"] = rec["cpu_baseline"]
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def cusparse_compare(workload: str, Ad, d_in, flush, steps: int, total_bytes: int):
    """The same call through torch.sparse (cuSPARSE) on the same device arrays, timed the
    same way; a comparison only, never part of the product path."""
    import torch

    try:
        Sp = torch.sparse_csr_tensor(Ad.indptr, Ad.indices, Ad.data, size=(Ad.rows, Ad.cols))
        if workload in SPMM_WORKLOADS:
            fn = lambda: torch.sparse.mm(Sp, d_in["B"])  # noqa: E731
            op = "torch.sparse.mm (cusparseSpMM)"
        elif workload == "c5-sddmm":
            Vt = d_in["V"].t()
            fn = lambda: torch.sparse.sampled_addmm(Sp, d_in["U"], Vt, beta=0.0, alpha=1.0)  # noqa: E731
            op = "torch.sparse.sampled_addmm (cusparseSDDMM; without the A.val product)"
        else:
            xx = d_in["x"]
            fn = lambda: torch.mv(Sp, xx)  # noqa: E731
            op = "torch.mv on a CSR tensor (cusparseSpMV)"
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        ts = []
        for _ in range(steps):
            if flush is not None:
                flush.zero_()
            a = torch.cuda.Event(enable_timing=True)
            b = torch.cuda.Event(enable_timing=True)
            a.record()
            fn()
            b.record()
            ts.append((a, b))
        torch.cuda.synchronize()
        ms = float(np.mean([a.elapsed_time(b) for a, b in ts]))
        return {"op": op, "ms_per_step": round(ms, 5), "value": round(total_bytes / (ms / 1e3) / 1e9, 2),
                "unit": "GB/s"}
    except Exception as exc:  # noqa: BLE001 -- a comparison must not fail the bench
        return {"error": str(exc)[:200]}


# ----------------------------------------------------------------------------- b200 arm
def main():
    args = parse()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        if args.workload != "c4":
            return run_matrix_reference(args, rank, world)
        return run_reference(args, rank, world)
    if args.workload != "c4":
        return run_matrix_workload(args, rank, world, local_rank)

    import torch
    import torch.distributed as dist

    from tilegen_b200 import lib, matrices as Mx
    from tilegen_b200.power import PowerIteration, uniform_bounds

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)

    n = args.rows
    bounds = uniform_bounds(n, world)
    r0, r1 = int(bounds[rank]), int(bounds[rank + 1])
    shard = Mx.c4_rows(r0, r1, n=n, per_row=C4_PER_ROW, seed=C4_SEED)
    x0_all = np.random.default_rng([X0_SEED, 0]).uniform(-1.0, 1.0, size=n)
    x0 = x0_all[r0:r1].copy()

    # pinned host copies (the e2e inputs)
    h_ip = torch.from_numpy(shard.indptr).pin_memory()
    h_ix = torch.from_numpy(shard.indices).pin_memory()
    h_d = torch.from_numpy(shard.data).pin_memory()
    h_x0 = torch.from_numpy(x0).pin_memory()
    h_xout = torch.empty(r1 - r0, dtype=torch.float64).pin_memory()
    h_lam = torch.empty(1, dtype=torch.float64).pin_memory()

    s = lib.default_schedule()
    s.threads_per_row, s.unroll, s.vector_width, s.block_size, s.tile = args.tpr, args.unroll, args.vec, args.block, 32
    s.split = lib.TG_SPLIT_STREAM if args.split == "stream" else lib.TG_SPLIT_ROWWISE
    lib.validate_schedule(s)

    d_ip = h_ip.to(dev)
    d_ix = h_ix.to(dev)
    d_d = h_d.to(dev)
    d_x0 = h_x0.to(dev)
    i32 = args.index_bits == 32 and args.split != "stream"
    pi = PowerIteration(d_ip, d_ix, d_d, bounds, rank, sched=s, index32=i32)
    if world > 1 and args.exchange in ("p2p", "ce"):
        pi.p2p_connect()
        pi.p2p_mode = "ce" if args.exchange == "ce" else "store"
        pi.ce_chunks = args.ce_chunks
    del d_ix
    x_out = torch.empty(r1 - r0, dtype=torch.float64, device=dev)
    lam = torch.empty(1, dtype=torch.float64, device=dev)
    stream = torch.cuda.current_stream(dev)

    kernel_events = []

    def one_step(record_kernels: bool):
        pi.set_x0(d_x0)
        if record_kernels:
            evs = []

            def on_step(i):
                e = torch.cuda.Event(enable_timing=True)
                e.record(stream)
                evs.append(e)

            pi.iterate(args.iters, on_step)
            kernel_events.append(evs)
        else:
            pi.iterate(args.iters)
        pi.result(x_out, lam)

    for _ in range(args.warmup):
        one_step(False)
    barrier()

    launches0 = pi.kernel_launches
    sampler = ClockSampler(local_rank) if rank == 0 else None
    if sampler:
        sampler.start()
    barrier()
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    wall0 = time.perf_counter()
    t_start.record(stream)
    for _ in range(args.steps):
        one_step(True)
    t_end.record(stream)
    barrier()
    wall = time.perf_counter() - wall0
    clocks = sampler.stop() if sampler else None
    launches = pi.kernel_launches - launches0
    ms_local = t_start.elapsed_time(t_end)
    kdur = [evs[2 * k].elapsed_time(evs[2 * k + 1]) for evs in kernel_events for k in range(args.iters)]
    k_ms_local = float(np.mean(kdur))

    # ---- random-gather floor of this shard's SpMV: the same gathers (this shard's own
    # column indices into the iterate) with nothing else.  The probe and this rank's
    # plain power-step kernel alternate, so both run at the same clocks (the SpMV is
    # clock-sensitive and the power cap moves the clock).
    from tilegen_b200 import bench_probe

    probe_out = torch.zeros(1, dtype=torch.float64, device=dev)

    def probe():
        bench_probe.gather_probe_f64(pi.indices.data_ptr(), pi.nnz, pi.x[0].data_ptr(), probe_out.data_ptr(),
                                     stream.cuda_stream, index32=pi.index32)

    def ev():
        return torch.cuda.Event(enable_timing=True)

    for _ in range(3):
        probe()
    pe, se = [], []
    for _ in range(10):
        a, b, c, d = ev(), ev(), ev(), ev()
        a.record(stream)
        probe()
        b.record(stream)
        c.record(stream)
        pi._gpu_step(pi.x[0], pi.shard(pi.x[1]))
        d.record(stream)
        pe.append((a, b))
        se.append((c, d))
    torch.cuda.synchronize(dev)
    gather_ms_local = float(np.median([a.elapsed_time(b) for a, b in pe]))
    step_ms_local = float(np.median([c.elapsed_time(d) for c, d in se]))

    # ---- e2e through the public API from pinned host buffers
    e2e_ms = []
    for it in range(args.e2e_steps + 1 if args.e2e_steps > 0 else 0):
        barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        ip = h_ip.to(dev, non_blocking=True)
        ix = h_ix.to(dev, non_blocking=True)
        dd = h_d.to(dev, non_blocking=True)
        xx = h_x0.to(dev, non_blocking=True)
        pe = PowerIteration(ip, ix, dd, bounds, rank, sched=s, index32=i32)
        if world > 1 and args.exchange in ("p2p", "ce"):
            pe.p2p_attach(pi.exchange_state)  # the mappings do not depend on the matrix
            pe.p2p_mode = pi.p2p_mode
            pe.ce_chunks = pi.ce_chunks
        del ix
        pe.set_x0(xx)
        pe.iterate(args.iters)
        xo, lo = pe.result()
        h_xout.copy_(xo, non_blocking=True)
        h_lam.copy_(lo, non_blocking=True)
        e1.record(stream)
        barrier()
        if it > 0:  # the first pass warms allocator and communicator buffers
            e2e_ms.append(e0.elapsed_time(e1))
        del pe, ip, dd, xx
    e2e_local = float(np.mean(e2e_ms)) if e2e_ms else float("nan")

    # ---- cuSPARSE SpMV on the same device arrays (N=1), a comparison only
    c4_cusparse = None
    if world == 1 and not args.no_cusparse:
        c4_cusparse = cusparse_c4(pi, n, dev, spmv_bytes(n, n, shard.nnz))

    # ---- the other BASELINE configurations (C1-C3 SpMV, C5 SpMM / SDDMM), each on its
    # own matrix, row-sharded over the same ranks
    workloads = {}
    if not args.no_workloads:
        peak, _ = measured_peaks()
        for wl in ("c1", "c2", "c3", "c5-spmm", "c5-sddmm") + (("c5-spmm-rcm", "blocked-spmm") if world == 1 else ()):
            rec = measure_matrix(wl, SCHEDULES[wl], args.steps, args.warmup, rank, world, dev, barrier, 2,
                                 want_cpu=(world == 1 and rank == 0 and not args.no_cpu_baseline),
                                 want_cusparse=(world == 1 and not args.no_cusparse), sample_clocks=False)
            v = torch.tensor([rec["ms_local"], rec["e2e_local"]], dtype=torch.float64, device=dev)
            if world > 1:
                dist.all_reduce(v, op=dist.ReduceOp.MAX)
            if rank == 0:
                d = summarise_matrix(rec, float(v[0].item()), world, peak)
                e2e_w = float(v[1].item())
                d["e2e"] = {"value": round(matrix_bytes(wl, rec["A"]) / (e2e_w / 1e3) / 1e9, 2), "unit": "GB/s",
                            "ms": round(e2e_w, 4), "h2d_bytes_per_step": rec["h2d"],
                            "d2h_bytes_per_step": rec["d2h"]}
                workloads[wl] = d
            del rec
            torch.cuda.empty_cache()

    # ---- max over ranks
    vals = torch.tensor([ms_local, k_ms_local, e2e_local], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(vals, op=dist.ReduceOp.MAX)
    ms_total, k_ms, e2e_step_ms = [float(v) for v in vals.cpu()]
    ms_step = ms_total / args.steps
    total_bytes = spmv_bytes(n, n, n * C4_PER_ROW)
    gbs = total_bytes * args.iters / (ms_step / 1e3) / 1e9
    e2e_gbs = total_bytes * args.iters / (e2e_step_ms / 1e3) / 1e9

    if rank == 0:
        peak, peak_kind = measured_peaks()
        local_bytes = spmv_bytes(r1 - r0, n, shard.nnz)
        achieved = local_bytes / (k_ms / 1e3) / 1e9
        kname = "spmv_stream_kernel(power)" if args.split == "stream" else (
            "power_p2p_kernel" if (world > 1 and args.exchange == "p2p") else "power_step_kernel")
        tr = traffic_record("c4_%d" % world, kname)
        # 32-byte L2 sectors per launch: one per x gather (uniform random columns) plus the
        # streamed arrays; the probe streams only the indices
        ib = 4 if pi.index32 else 8
        probe_sectors = shard.nnz + shard.nnz * ib / 32
        step_sectors = shard.nnz + (shard.nnz * (ib + 8) + (r1 - r0 + 1) * 8 + (r1 - r0) * 8) / 32
        roofline = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                    "frac": round(achieved / peak, 4), "peak_source": peak_kind + " (MEASURED_PEAKS.json hbm_gbs)"
                    if peak_kind == "measured" else "fallback 6.65 TB/s",
                    "kernel": kname, "kernel_ms": round(k_ms, 4),
                    "algorithmic_bytes_per_launch": local_bytes,
                    "traffic": tr["dram_bytes_per_launch"] if tr else None,
                    "gather_floor": {
                        "ms": round(gather_ms_local, 4),
                        "gathers_per_s": round(shard.nnz / (gather_ms_local / 1e3), 1),
                        "step_ms": round(step_ms_local, 4),
                        "frac": round(gather_ms_local / step_ms_local, 4),
                        "l2_sectors_probe": int(probe_sectors),
                        "l2_sectors_step": int(step_sectors),
                        "sector_rate_frac": round((step_sectors / step_ms_local) / (probe_sectors / gather_ms_local),
                                                  4),
                        "what": "rank 0: tg_gather_probe_f64 on the shard's own column indices (the "
                                "SpMV's x gathers alone, same load path and L2 policy) alternated with "
                                "the plain power-step kernel; frac = probe time / step-kernel time; "
                                "sector_rate_frac = the step's 32-byte L2 sectors per second (one per "
                                "gather plus its streamed indices, values, row offsets and output) over "
                                "the probe's (one per gather plus its indices)"}}
        line = {
            "metric": "effective_hbm_gbs_power_iteration_spmv",
            "value": round(gbs, 2),
            "unit": "GB/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms_step, 4),
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": "f64",
            "data": "synthetic (seeded C4 generator, values U(-1,1))",
            "config": workload_config(n, world, args.exchange),
            "e2e": {"value": round(e2e_gbs, 2), "unit": "GB/s",
                    "h2d_bytes_per_step": int(h_ip.numel() * 8 + h_ix.numel() * 8 + h_d.numel() * 8 + h_x0.numel() * 8),
                    "d2h_bytes_per_step": int(h_xout.numel() * 8 + 8), "ms_per_step": round(e2e_step_ms, 3)},
            "gpu_launches": int(launches),
            "roofline": roofline,
            "clocks": clocks,
            "wall_s_timed": round(wall, 4),
            "schedule": {"split": args.split, "tpr": args.tpr, "unroll": args.unroll, "vec": args.vec,
                         "block": args.block, "column_index_bits": 32 if pi.index32 else 64},
            "lambda": float(lam[0].item()),  # the timed steps' result (rank 0's copy)
        }
        if world > 1:
            # communication broken out per iteration: the timed iteration (with its
            # exchange, max over ranks) against rank 0's compute-only step kernel timed
            # beside the gather probe, and the iterate bytes rank 0 receives
            it_ms = ms_step / args.iters
            line["comm"] = {"iteration_ms": round(it_ms, 4), "compute_only_ms": round(step_ms_local, 4),
                            "exchange_ms": round(max(it_ms - step_ms_local, 0.0), 4),
                            "received_bytes_per_iteration": int(8 * (n - (r1 - r0))),
                            "exchange": args.exchange}
        if c4_cusparse is not None:
            c4_cusparse["vs_cusparse"] = (round(c4_cusparse["ms_per_spmv"] / k_ms, 3)
                                          if "ms_per_spmv" in c4_cusparse else None)
            line["cusparse"] = c4_cusparse
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(shard, x0_all)
        if workloads:
            line["workloads"] = workloads
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def cusparse_c4(pi, n: int, dev, nbytes: int, reps: int = 10):
    """cuSPARSE SpMV (torch.mv on a CSR tensor) on the power iteration's own arrays (one
    GPU: the padded layout is the identity), timed per call with CUDA events; compared
    with the fused power-step kernel, which does the SpMV plus the norm."""
    import torch

    try:
        # cuSPARSE needs row offsets and column indices of one type: the power iteration
        # keeps its columns as int32, so the comparison gets an int64 copy
        cols = pi.indices if pi.indices.dtype == pi.indptr.dtype else pi.indices.to(pi.indptr.dtype)
        if cols.dtype != pi.indptr.dtype or cols.numel() != pi.nnz:
            raise ValueError("index arrays of the comparison do not match")
        Sp = torch.sparse_csr_tensor(pi.indptr, cols, pi.data, size=(n, n))
        x = pi.x[0][:n].clone()
        for _ in range(3):
            torch.mv(Sp, x)
        torch.cuda.synchronize(dev)
        ts = []
        for _ in range(reps):
            a = torch.cuda.Event(enable_timing=True)
            b = torch.cuda.Event(enable_timing=True)
            a.record()
            torch.mv(Sp, x)
            b.record()
            ts.append((a, b))
        torch.cuda.synchronize(dev)
        ms = float(np.mean([a.elapsed_time(b) for a, b in ts]))
        return {"op": "torch.mv on a CSR tensor (cusparseSpMV), same arrays, inputs larger than L2",
                "ms_per_spmv": round(ms, 4), "value": round(nbytes / (ms / 1e3) / 1e9, 2), "unit": "GB/s"}
    except Exception as exc:  # noqa: BLE001 -- a comparison must not fail the bench
        return {"error": str(exc)[:200]}


def cpu_baseline(A, x0):
    spmv, kind, desc, threads = cpu_reference_spmv(A, A.cols)
    iters = 3
    cpu_power_sample(A, x0, 1, spmv)
    sec = cpu_power_sample(A, x0, iters, spmv)
    gbs = spmv_bytes(A.rows, A.cols, A.nnz) * iters / sec / 1e9
    return {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": kind,
            "sample": "%d of the %d power iterations on the full matrix (%d rows, %d nnz), host cores"
                      % (iters, ITERS, A.rows, A.nnz), "impl": desc}


if __name__ == "__main__":
    sys.exit(main())
