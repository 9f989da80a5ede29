"""Schedule autotuner for the b200 backend (mirror of tilegen/autotune.py).

Same surface as the reference tuner: a discrete search space over the schedule knobs
(``SEARCH_SPACE``, tilegen/autotune.py:47-53), illegal combinations pruned with logged
reasons (``illegal_reason`` / ``enumerate_configs`` / ``legal_configs`` / ``prune_log``,
:59-93), random or coordinate-descent candidate selection seeded at the fixed naive
``BASELINE`` (:196-222), ``tune`` returning every variant with its timings, error and
speedup (:225-335) and ``write_outputs`` writing the compact and the full summaries in
the reference's schema (:338-417).

What is b200-specific:

* the candidates can also vary the row mapping (``splits``: the reference's rowwise
  T/TPR mapping, the nnz-balanced merge split, the streaming SpMV); a config's split is
  part of its hash, so the reference's cache keys are unchanged for rowwise configs;
* every variant runs on the GPU through the library's C ABI on device buffers that are
  allocated once, and is timed with CUDA events on the launching stream (the
  reference times host wall clock around a synchronising call, :182-190); by default
  a buffer larger than L2 is written between timed calls, so each call starts cold;
* each variant is verified before it is timed with the reference's acceptance rule
  (``8 * eps * max_row_nnz * max|ref| + 1e-12``, :271-277) and additionally reports
  the max relative error with the floored denominator;
* ``bandwidth_gbs`` keeps the reference's traffic model (:96-110) so the numbers are
  comparable with its tables; ``effective_gbs`` uses the compulsory bytes (each
  operand read once: indptr + indices + values + dense inputs + outputs), which is the
  figure compared against the HBM roofline.
"""

from __future__ import annotations

import argparse
import itertools
import json
import os
import random
import statistics
from typing import Any, Dict, List, Optional, Sequence, Tuple

import numpy as np

from . import codegen as _codegen
from . import lib as _lib
from .codegen import Config
from .matrices import CSR
from .verify import inputs_for, load_matrix, reference, tolerance

__all__ = [
    "SEARCH_SPACE",
    "B200_SEARCH_SPACE",
    "SPLITS",
    "BASELINE",
    "illegal_reason",
    "enumerate_configs",
    "legal_configs",
    "prune_log",
    "flops_bytes",
    "tune",
    "write_outputs",
]

# The reference's discrete space (4 * 5 * 4 * 3 * 3 = 720 raw combinations).
SEARCH_SPACE: Dict[str, List[int]] = {
    "tile_size": [32, 64, 128, 256],
    "threads_per_row": [1, 2, 4, 8, 32],
    "unroll": [1, 2, 4, 8],
    "vector_width": [1, 2, 4],
    "block_size": [128, 256, 512],
}

# The b200 templates are also instantiated for 16 lanes per row.
B200_SEARCH_SPACE: Dict[str, List[int]] = dict(SEARCH_SPACE, threads_per_row=[1, 2, 4, 8, 16, 32])

# Row mappings of the b200 kernels ("stream" is a distinct kernel only for SpMV).
SPLITS: Tuple[str, ...] = ("rowwise", "merge", "stream", "block")

BASELINE = Config(tile_size=32, threads_per_row=1, unroll=1, vector_width=1, block_size=128)

_SUPPORTED_TPR = (1, 2, 4, 8, 16, 32)
_STREAM_KERNELS = ("spmv", "fused_spmv_axpy")
# the block split (row groups sharing a column list) is an SpMM mapping; elsewhere it
# would repeat the merge split's candidates
_BLOCK_KERNELS = ("spmm",)


def illegal_reason(cfg: Config) -> Optional[str]:
    """Reason a config is illegal, or None.  The first four rules are the reference's
    (tilegen/autotune.py:59-72), kept so that the prune log matches it; the rest are
    limits of the b200 templates."""
    if cfg.threads_per_row > cfg.block_size:
        return "threads_per_row (%d) > block_size (%d)" % (cfg.threads_per_row, cfg.block_size)
    if cfg.block_size % cfg.threads_per_row != 0:
        return "block_size (%d) not divisible by threads_per_row (%d)" % (cfg.block_size, cfg.threads_per_row)
    if cfg.vector_width > cfg.unroll:
        return "vector_width (%d) > unroll (%d) (unsound: no unroll slots)" % (cfg.vector_width, cfg.unroll)
    if cfg.vector_width not in (1, 2, 4):
        return "vector_width %d not supported" % cfg.vector_width
    if cfg.threads_per_row not in _SUPPORTED_TPR:
        return "threads_per_row %d has no b200 instance (1, 2, 4, 8, 16, 32)" % cfg.threads_per_row
    if cfg.unroll not in (1, 2, 4, 8):
        return "unroll %d has no b200 instance (1, 2, 4, 8)" % cfg.unroll
    if cfg.block_size % 32 != 0 or not 32 <= cfg.block_size <= 512:
        return "block_size %d is not a multiple of 32 in [32, 512]" % cfg.block_size
    if cfg.split not in SPLITS and cfg.split != "auto":
        return "split %r unknown" % cfg.split
    return None


def enumerate_configs(space: Optional[Dict[str, List[int]]] = None,
                      splits: Sequence[str] = ("rowwise",)) -> List[Tuple[Config, Optional[str]]]:
    """All raw configs of ``space`` (default: the reference's) x ``splits``, each with
    its prune reason (None == legal)."""
    space = space or SEARCH_SPACE
    keys = list(space.keys())
    out = []
    for split in splits:
        for combo in itertools.product(*(space[k] for k in keys)):
            cfg = Config(**dict(zip(keys, combo)), split=split)
            out.append((cfg, illegal_reason(cfg)))
    return out


def legal_configs(space: Optional[Dict[str, List[int]]] = None, splits: Sequence[str] = ("rowwise",)) -> List[Config]:
    return [cfg for cfg, reason in enumerate_configs(space, splits) if reason is None]


def prune_log(space: Optional[Dict[str, List[int]]] = None, splits: Sequence[str] = ("rowwise",)) -> List[Dict[str, str]]:
    return [{"config": str(cfg.to_dict()), "reason": reason}
            for cfg, reason in enumerate_configs(space, splits) if reason is not None]


# --------------------------------------------------------------------------- traffic
def flops_bytes(kernel: str, A: CSR, K: int, dtype: str = "f64") -> Tuple[float, float, float]:
    """(FLOPs, reference-model bytes, compulsory bytes) of one call.

    The reference model (tilegen/autotune.py:96-110) counts 8-byte values and one dense
    element per nonzero; the compulsory bytes count every operand once with the value
    size of ``dtype`` and 8-byte indices."""
    M, N = A.shape
    nnz = float(A.nnz)
    e = 8.0 if dtype == "f64" else 4.0
    csr = (M + 1) * 8.0 + nnz * 8.0 + nnz * e
    if kernel == "spmv":
        return 2.0 * nnz, nnz * 16.0 + (M + 1) * 8.0 + nnz * 8.0 + M * 8.0, csr + (N + M) * e
    if kernel == "spmm":
        return 2.0 * nnz * K, nnz * 16.0 + (M + 1) * 8.0 + nnz * K * 8.0 + M * K * 8.0, csr + (N + M) * K * e
    if kernel == "sddmm":
        return (2.0 * nnz * K, nnz * 16.0 + (M + 1) * 8.0 + 2.0 * nnz * K * 8.0 + nnz * 8.0,
                csr + (M + N) * K * e + nnz * e)
    if kernel == "fused_spmv_axpy":
        return 2.0 * nnz, nnz * 16.0 + (M + 1) * 8.0 + nnz * 8.0 + 2 * M * 8.0, csr + (N + 2 * M) * e
    if kernel == "axpy":
        return 2.0 * M, 3.0 * M * 8.0, 3.0 * M * e
    raise ValueError(kernel)


# --------------------------------------------------------------------------- device calls
class _DeviceCase:
    """Device copies of one (kernel, matrix, inputs) case, allocated once; ``call(gen)``
    runs one variant through the library's C ABI on the current stream."""

    def __init__(self, kernel: str, A: CSR, data, K: int, dtype: str):
        import torch

        from . import device as D

        self.torch = torch
        self.D = D
        self.kernel = kernel
        self.dt = torch.float64 if dtype == "f64" else torch.float32
        dev = torch.device("cuda", torch.cuda.current_device())
        self.dev = dev
        x, w, B, U, V, alpha, beta = data
        T = lambda a: torch.as_tensor(np.ascontiguousarray(a)).to(dev, dtype=self.dt)  # noqa: E731
        self.alpha, self.beta = alpha, beta
        self.x, self.w = T(x), T(w)
        if kernel != "axpy":
            self.A = D.DeviceCSR.from_host(A, dev, self.dt)
        if kernel == "spmm":
            self.B = T(B)
            self.out = torch.zeros((A.rows, K), dtype=self.dt, device=dev)
        elif kernel == "sddmm":
            self.U, self.V = T(U), T(V)
            self.out = torch.zeros(A.nnz, dtype=self.dt, device=dev)
        else:
            self.out = torch.zeros(A.rows, dtype=self.dt, device=dev)

    def call(self, gen) -> None:
        # workspaces come from the wrappers' per-device cache (grown before timing starts)
        D, k = self.D, self.kernel
        if k == "spmv":
            D.spmv(self.A, self.x, self.out, sched=gen)
        elif k == "fused_spmv_axpy":
            D.fused_spmv_axpy(self.A, self.x, self.w, self.alpha, self.beta, z=self.out, sched=gen)
        elif k == "spmm":
            D.spmm(self.A, self.B, self.out, sched=gen)
        elif k == "sddmm":
            D.sddmm(self.A, self.U, self.V, self.out, sched=gen)
        elif k == "axpy":
            D.axpy(self.x, self.w, self.alpha, self.beta, z=self.out, sched=gen)
        else:
            raise ValueError(k)

    def result(self) -> np.ndarray:
        self.torch.cuda.synchronize(self.dev)
        return self.out.double().cpu().numpy().ravel()


def time_events(fn, warmup: int, iters: int, flush=None) -> Tuple[float, float, float]:
    """(mean, min, median) milliseconds of ``fn`` with one CUDA event pair per call on
    the current stream; ``flush`` (a device buffer larger than L2) is rewritten before
    each timed call."""
    import torch

    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    times = []
    for _ in range(iters):
        if flush is not None:
            flush.zero_()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        b.synchronize()
        times.append(a.elapsed_time(b))
    return sum(times) / len(times), min(times), statistics.median(times)


# --------------------------------------------------------------------------- tuning
def _candidate_configs(budget: int, mode: str, rng: random.Random, kernel: str = "spmv",
                       splits: Sequence[str] = ("rowwise",), space: Optional[Dict[str, List[int]]] = None,
                       dtype: str = "f64") -> List[Config]:
    """The reference's selection (tilegen/autotune.py:196-222) over ``space`` x ``splits``;
    the baseline is always first.  Stream variants are kept only for the SpMV kernels
    (for SpMM/SDDMM the stream split is the merge kernel)."""
    space = space or SEARCH_SPACE
    splits = [s for s in splits if (s != "stream" or kernel in _STREAM_KERNELS) and
              (s != "block" or kernel in _BLOCK_KERNELS)]
    base = Config(**dict(BASELINE.to_dict(), dtype=dtype))
    if mode == "coordinate":
        best = base
        chosen = [best]
        seen = {best.hash()}
        for key in ["tile_size", "threads_per_row", "unroll", "vector_width", "block_size"]:
            for value in space[key]:
                cand = Config(**dict(best.to_dict(), **{key: value}))
                if illegal_reason(cand) is None and cand.hash() not in seen:
                    chosen.append(cand)
                    seen.add(cand.hash())
                    if len(chosen) >= budget:
                        return chosen
        for split in splits:
            if split == "rowwise":
                continue
            cand = Config(**dict(best.to_dict(), split=split))
            if cand.hash() not in seen and len(chosen) < budget:
                chosen.append(cand)
                seen.add(cand.hash())
        return chosen[:budget]
    pool = [Config(**dict(c.to_dict(), dtype=dtype)) for c in legal_configs(space, splits)]
    pool = [c for c in pool if c.hash() != base.hash()]
    rng.shuffle(pool)
    out = [base]
    for c in pool:
        if len(out) >= budget:
            break
        out.append(c)
    return out


def tune(
    kernel_name: str,
    matrix,
    budget: int = 40,
    mode: str = "random",
    backend: str = "b200",
    K: int = 8,
    workdir: Optional[str] = None,
    warmup: int = 5,
    iters: int = 25,
    seed: int = 0,
    splits: Sequence[str] = SPLITS,
    space: Optional[Dict[str, List[int]]] = None,
    dtype: str = "f64",
    flush_l2: bool = True,
) -> Dict[str, Any]:
    """Autotune one (kernel, matrix) pair on the current GPU; returns every variant tried
    (the reference's result schema, tilegen/autotune.py:319-335)."""
    if backend != "b200":
        raise ValueError("this tuner drives the 'b200' backend (got %r)" % backend)
    import torch

    _lib.load()
    rng = random.Random(seed)
    A, class_name = load_matrix(matrix)
    data = inputs_for(kernel_name, A, K, seed)
    ref = np.asarray(reference(kernel_name, A, data), dtype=np.float64).ravel()
    flops, nbytes, cbytes = flops_bytes(kernel_name, A, K, dtype)
    M, N = A.shape
    case = _DeviceCase(kernel_name, A, data, K, dtype)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=case.dev) if flush_l2 else None
    tol = tolerance(A, ref, dtype)
    base_cfg = Config(**dict(BASELINE.to_dict(), dtype=dtype))

    records: List[Dict[str, Any]] = []
    baseline_ms: Optional[float] = None
    for cfg in _candidate_configs(budget, mode, rng, kernel_name, splits, space, dtype):
        rec: Dict[str, Any] = {"kernel": kernel_name, "matrix_class": class_name, "rows": int(M), "nnz": int(A.nnz),
                               "config": cfg.to_dict(), "skipped": None}
        gen = _codegen.generate(kernel_name, cfg, backend, outdir=workdir, write=bool(workdir))
        try:
            _, log = _codegen.compile_generated(gen, backend)
            case.out.zero_()
            case.call(gen)
            outv = case.result()
            ms_mean, ms_min, ms_median = time_events(lambda: case.call(gen), warmup, iters, flush)
        except _lib.TgError as exc:
            rec["skipped"] = "kernel error: %s" % exc
            records.append(rec)
            continue
        diff = np.abs(outv - ref)
        max_abs = float(diff.max()) if diff.size else 0.0
        scale = float(np.abs(ref).max()) if ref.size else 0.0
        max_rel = float((diff / np.maximum(np.abs(ref), max(1e-3 * scale, 1e-300))).max()) if diff.size else 0.0
        rec.update({
            "ms_mean": ms_mean,
            "ms_min": ms_min,
            "ms_median": ms_median,
            "gflops": flops / (ms_min * 1e6) if ms_min > 0 else 0.0,
            "bandwidth_gbs": nbytes / (ms_min * 1e6) if ms_min > 0 else 0.0,
            "effective_gbs": cbytes / (ms_median * 1e6) if ms_median > 0 else 0.0,
            "max_abs_err": max_abs,
            "max_rel_err": max_rel,
            "tolerance": tol,
            "ok": bool(max_abs <= tol),
            "cold_l2": bool(flush_l2),
            "log": log,
        })
        if cfg.hash() == base_cfg.hash():
            baseline_ms = ms_min
        records.append(rec)

    base = baseline_ms
    if base is None:
        measured = [r for r in records if r.get("ms_min")]
        base = measured[0]["ms_min"] if measured else None
    for r in records:
        r["speedup_vs_naive"] = (base / r["ms_min"]) if (r.get("ms_min") and base) else None
    measured = [r for r in records if r.get("ms_min") and r.get("ok")]
    winner = min(measured, key=lambda r: r["ms_median"]) if measured else None
    return {
        "kernel": kernel_name,
        "matrix_class": class_name,
        "baseline": base_cfg.to_dict(),
        "baseline_ms_min": base,
        "winner": winner["config"] if winner else None,
        "winner_metrics": winner if winner else None,
        "records": records,
    }


# --------------------------------------------------------------------------- outputs
_METRIC_FIELDS = ["ms_mean", "ms_min", "ms_median", "gflops", "bandwidth_gbs", "effective_gbs", "max_abs_err",
                  "max_rel_err", "tolerance", "ok", "speedup_vs_naive"]

_CSV_COLS = ["matrix_class", "kernel", "split", "tile_size", "threads_per_row", "unroll", "vector_width",
             "block_size", "ms_mean", "ms_min", "ms_median", "gflops", "bandwidth_gbs", "effective_gbs",
             "max_abs_err", "ok", "speedup_vs_naive"]


def _compact_metrics(record: Optional[Dict[str, Any]]) -> Optional[Dict[str, Any]]:
    if record is None:
        return None
    return {key: record.get(key) for key in _METRIC_FIELDS if key in record}


def _flat_row(record: Dict[str, Any]) -> Dict[str, Any]:
    row = {"matrix_class": record["matrix_class"], "kernel": record["kernel"]}
    row.update(record["config"])
    row.update({key: record.get(key) for key in _METRIC_FIELDS if key in record})
    return row


def _write_csv(path: str, rows: List[Dict[str, Any]]) -> None:
    with open(path, "w") as fh:
        fh.write(",".join(_CSV_COLS) + "\n")
        for row in rows:
            fh.write(",".join(str(row.get(c, "")) for c in _CSV_COLS) + "\n")


def write_outputs(all_results: List[Dict[str, Any]], outdir: str, env: Dict[str, Any], pruned: List[Dict[str, str]],
                  full_outdir: str = "build") -> None:
    """Compact summary (per-pair winners, top five per class) to ``outdir`` and the full
    sweep to ``full_outdir``, in the reference's files and schema
    (tilegen/autotune.py:338-417)."""
    os.makedirs(outdir, exist_ok=True)
    os.makedirs(full_outdir, exist_ok=True)
    best: Dict[str, Dict[str, Any]] = {}
    flat: List[Dict[str, Any]] = []
    compact: List[Dict[str, Any]] = []
    top5: Dict[str, List[Dict[str, Any]]] = {}
    for res in all_results:
        cls = res["matrix_class"]
        compact.append({"kernel": res["kernel"], "matrix_class": cls, "baseline": res["baseline"],
                        "baseline_ms_min": res["baseline_ms_min"], "winner": res["winner"],
                        "winner_metrics": _compact_metrics(res["winner_metrics"])})
        best.setdefault(cls, {})[res["kernel"]] = {"config": res["winner"],
                                                   "metrics": _compact_metrics(res["winner_metrics"]),
                                                   "baseline_ms_min": res["baseline_ms_min"]}
        for r in res["records"]:
            if r.get("ms_min") is not None:
                flat.append(_flat_row(r))
                if r.get("ok"):
                    top5.setdefault(cls, []).append(_flat_row(r))
    for cls in top5:
        top5[cls] = sorted(top5[cls], key=lambda r: r["ms_median"])[:5]
    with open(os.path.join(full_outdir, "autotune.json"), "w") as fh:
        json.dump({"hardware": env, "baseline": BASELINE.to_dict(), "search_space": SEARCH_SPACE,
                   "splits": list(SPLITS), "pruned": pruned, "results": all_results}, fh, indent=2)
    _write_csv(os.path.join(full_outdir, "autotune.csv"), flat)
    with open(os.path.join(outdir, "autotune.json"), "w") as fh:
        json.dump({"hardware": env, "baseline": BASELINE.to_dict(), "search_space": SEARCH_SPACE,
                   "splits": list(SPLITS), "pruned": pruned, "results": compact, "best": best, "top5": top5},
                  fh, indent=2)
    with open(os.path.join(outdir, "best_configs.json"), "w") as fh:
        json.dump(best, fh, indent=2)
    _write_csv(os.path.join(outdir, "autotune.csv"), [row for cls in sorted(top5) for row in top5[cls]])


def hardware() -> Dict[str, Any]:
    """The device the sweep ran on (name, SMs, memory, library version)."""
    import torch

    p = torch.cuda.get_device_properties(torch.cuda.current_device())
    return {"backend": "b200", "device": p.name, "sms": p.multi_processor_count,
            "memory_gb": round(p.total_memory / 1e9, 1), "library": _lib.version(), "torch": torch.__version__}


def main(argv=None) -> int:
    """``python -m tilegen_b200.autotune``: the reference's scripts/autotune.py loop for
    the b200 backend over the BASELINE classes (c1..c5) or reference corpus classes."""
    from . import matrices as _m

    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--budget", type=int, default=40)
    ap.add_argument("--out", default="autotune_results")
    ap.add_argument("--full-out", default="build")
    ap.add_argument("--mode", default="random", choices=["random", "coordinate"])
    ap.add_argument("--kernels", default="spmv")
    ap.add_argument("--classes", default="c1,c2,c3")
    ap.add_argument("--splits", default=",".join(SPLITS))
    ap.add_argument("--dtype", default="f64", choices=["f64", "f32"])
    ap.add_argument("--K", type=int, default=8)
    ap.add_argument("--iters", type=int, default=25)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--warm-l2", action="store_true", help="do not flush L2 between timed calls")
    args = ap.parse_args(argv)
    splits = [s for s in args.splits.split(",") if s]
    results = []
    for cls in [c for c in args.classes.split(",") if c]:
        m = _m.baseline_matrix(cls) if cls in _m.baseline_configs() else _m.make_matrix(cls)
        for kernel in [k for k in args.kernels.split(",") if k]:
            res = tune(kernel, m, budget=args.budget, mode=args.mode, K=args.K, warmup=args.warmup, iters=args.iters,
                       splits=splits, space=B200_SEARCH_SPACE, dtype=args.dtype, flush_l2=not args.warm_l2)
            results.append(res)
            w, wm = res["winner"], res["winner_metrics"]
            if w:
                print("%-20s %-16s winner %s T=%d TPR=%d U=%d V=%d B=%d  %.4f ms  %.0f GB/s  %.2fx" % (
                    cls, kernel, w["split"], w["tile_size"], w["threads_per_row"], w["unroll"], w["vector_width"],
                    w["block_size"], wm["ms_median"], wm["effective_gbs"], wm["speedup_vs_naive"] or 0.0))
            else:
                print("%-20s %-16s no verified variant" % (cls, kernel))
    write_outputs(results, args.out, hardware(), prune_log(B200_SEARCH_SPACE, splits), full_outdir=args.full_out)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
