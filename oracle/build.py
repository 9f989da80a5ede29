"""Build recipe for the parity oracle (TEST INFRASTRUCTURE ONLY).

* ``oracle/_build/liboracle.so`` -- the plain-C restatement in ``tg_oracle.c``
  (gcc, ``-ffp-contract=off`` so products and sums round exactly as the serial
  reference's do).  Built here and on the GPU box alike.
* ``oracle/_ref/libtgref.so`` -- the reference's own serial kernels, compiled from
  ``cpp/src/ref.cpp`` where it lies in the reference tree, plus ``ref_shim.cpp``.
* ``oracle/_ref/ref_omp_<kernel>_<dtype>_<cfg>.so`` -- the reference's OpenMP backend:
  the reference's code generator (``tilegen.codegen.generate(..., "cpu")``) is imported
  from the reference tree, its emitted C++ is written to ``oracle/_ref/gen/`` and
  compiled with the reference's OpenMP flags (tilegen/verify.py:238-247) except that
  ``-march=native`` becomes ``-march=x86-64-v3``, because the objects are built in this
  container and run on the GPU box's host.  ``rebuild_ref_native()`` recompiles the
  emitted sources with ``-march=native`` on the machine that runs them (the bench's
  reference arm does that when a compiler is present).

The ``_ref`` outputs need the reference tree, which only exists in the build container;
they are git-ignored and travel to the GPU box with the working tree.
"""

from __future__ import annotations

import glob
import json
import os
import shutil
import subprocess
import sys
from typing import Dict, List, Optional

ORACLE_DIR = os.path.dirname(os.path.abspath(__file__))
BUILD_DIR = os.path.join(ORACLE_DIR, "_build")
REF_DIR = os.path.join(ORACLE_DIR, "_ref")
GEN_DIR = os.path.join(REF_DIR, "gen")
ORACLE_LIB = os.path.join(BUILD_DIR, "liboracle.so")
TGREF_LIB = os.path.join(REF_DIR, "libtgref.so")
# The reference checkout: $TILEGEN_REFERENCE_ROOT, else a `reference` directory beside
# this repository's root (the layout of a source checkout of both projects).
DEFAULT_REF_ROOT = os.environ.get("TILEGEN_REFERENCE_ROOT",
                                  os.path.join(os.path.dirname(os.path.dirname(ORACLE_DIR)), "reference"))

# CPU schedules emitted for the reference OpenMP backend: the reference default
# (tilegen/autotune.py:55-56) and two tiled/unrolled variants its CPU autotune explores
# (tile_size and unroll change the emitted OpenMP code, tilegen/codegen.py:414-530).
# vector_width stays 1: with vector_width > 1 and unroll > 1 the reference's SpMM emitter
# places `#pragma omp simd` before a declaration (tilegen/codegen.py:488-492), which g++
# rejects, so those points of its space do not compile.
REF_CPU_CONFIGS: Dict[str, Dict[str, int]] = {
    "T32U1": dict(tile_size=32, threads_per_row=1, unroll=1, vector_width=1, block_size=128),
    "T64U2": dict(tile_size=64, threads_per_row=1, unroll=2, vector_width=1, block_size=128),
    "T128U4": dict(tile_size=128, threads_per_row=1, unroll=4, vector_width=1, block_size=512),
}
REF_KERNELS_F64 = ["spmv", "spmm", "sddmm", "fused_spmv_axpy", "axpy"]
REF_KERNELS_F32 = ["spmv", "spmm", "sddmm", "fused_spmv_axpy", "axpy"]


def _run(cmd: List[str]) -> None:
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError("command failed: %s\n%s%s" % (" ".join(cmd), res.stdout, res.stderr))


def _stale(target: str, deps: List[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build_oracle(force: bool = False) -> str:
    os.makedirs(BUILD_DIR, exist_ok=True)
    src = os.path.join(ORACLE_DIR, "tg_oracle.c")
    if force or _stale(ORACLE_LIB, [src]):
        cc = shutil.which("gcc") or shutil.which("cc")
        if cc is None:
            raise RuntimeError("no C compiler for the oracle")
        _run([cc, "-O2", "-ffp-contract=off", "-fopenmp", "-fPIC", "-shared", "-o", ORACLE_LIB, src, "-lm"])
    return ORACLE_LIB


def _ref_kernel(ref_dsl, name: str, dtype: str):
    """The reference's standard kernel `name` (tilegen/dsl.py:214-256) with every tensor
    declared as `dtype` (the f32 path of tilegen/dsl.py:124-147)."""
    d = ref_dsl
    i, j, k = d.Index("i"), d.Index("j"), d.Index("k")
    M, N, K = "M", "N", "K"
    if name == "spmv":
        A = d.sparse_tensor("A", d.CSR, shape=(M, N), dtype=dtype)
        x = d.dense_tensor("x", shape=(N,), dtype=dtype)
        y = d.dense_tensor("y", shape=(M,), dtype=dtype)
        return d.kernel("spmv", [d.assign(y[i], d.reduce_sum(j, A[i, j] * x[j]))])
    if name == "spmm":
        A = d.sparse_tensor("A", d.CSR, shape=(M, N), dtype=dtype)
        B = d.dense_tensor("B", shape=(N, K), dtype=dtype)
        C = d.dense_tensor("C", shape=(M, K), dtype=dtype)
        return d.kernel("spmm", [d.assign(C[i, k], d.reduce_sum(j, A[i, j] * B[j, k]))])
    if name == "sddmm":
        A = d.sparse_tensor("A", d.CSR, shape=(M, N), dtype=dtype)
        U = d.dense_tensor("U", shape=(M, K), dtype=dtype)
        V = d.dense_tensor("V", shape=(N, K), dtype=dtype)
        C = d.sparse_tensor("C", d.CSR, shape=(M, N), dtype=dtype)
        return d.kernel("sddmm", [d.assign(C[i, j], A[i, j] * d.reduce_sum(k, U[i, k] * V[j, k]))])
    if name == "fused_spmv_axpy":  # tilegen/dsl.py:237-247
        A = d.sparse_tensor("A", d.CSR, shape=(M, N), dtype=dtype)
        x = d.dense_tensor("x", shape=(N,), dtype=dtype)
        w = d.dense_tensor("w", shape=(M,), dtype=dtype)
        z = d.dense_tensor("z", shape=(M,), dtype=dtype)
        alpha = d.scalar_tensor("alpha", dtype=dtype)
        beta = d.scalar_tensor("beta", dtype=dtype)
        t = d.dense_tensor("t", shape=(M,), dtype=dtype)
        return d.kernel("fused_spmv_axpy", [d.assign(t[i], d.reduce_sum(j, A[i, j] * x[j])),
                                            d.assign(z[i], alpha * t[i] + beta * w[i])])
    if name == "axpy":  # tilegen/dsl.py:250-256
        x = d.dense_tensor("x", shape=(M,), dtype=dtype)
        w = d.dense_tensor("w", shape=(M,), dtype=dtype)
        z = d.dense_tensor("z", shape=(M,), dtype=dtype)
        alpha = d.scalar_tensor("alpha", dtype=dtype)
        beta = d.scalar_tensor("beta", dtype=dtype)
        return d.kernel("axpy", [d.assign(z[i], alpha * x[i] + beta * w[i])])
    raise ValueError(name)


def build_ref(ref_root: str = DEFAULT_REF_ROOT, force: bool = False) -> Dict[str, str]:
    """Build libtgref.so and the reference OpenMP kernels; returns {name: path}.

    Returns an empty dict when the reference tree is absent (e.g. on the GPU box)."""
    out: Dict[str, str] = {}
    ref_cpp = os.path.join(ref_root, "cpp", "src", "ref.cpp")
    if not os.path.exists(ref_cpp):
        return out
    os.makedirs(GEN_DIR, exist_ok=True)
    cxx = shutil.which("g++") or shutil.which("c++")
    if cxx is None:
        raise RuntimeError("no C++ compiler for the reference build")
    shim = os.path.join(ORACLE_DIR, "ref_shim.cpp")
    if force or _stale(TGREF_LIB, [ref_cpp, shim]):
        _run([cxx, "-std=c++17", "-O2", "-ffp-contract=off", "-fPIC", "-shared",
              "-I" + os.path.join(ref_root, "cpp", "include"), "-o", TGREF_LIB, ref_cpp, shim])
    out["tgref"] = TGREF_LIB

    sys.path.insert(0, ref_root)
    try:
        from tilegen import codegen as ref_codegen  # noqa: E402  (reference tree)
        from tilegen import dsl as ref_dsl  # noqa: E402
    finally:
        sys.path.pop(0)
    manifest = {}
    for dtype, names in (("f64", REF_KERNELS_F64), ("f32", REF_KERNELS_F32)):
        std = ref_dsl.standard_kernels()
        for name in names:
            kern = std[name] if dtype == "f64" else _ref_kernel(ref_dsl, name, "f32")
            for cfg_name, knobs in REF_CPU_CONFIGS.items():
                cfg = ref_codegen.Config(dtype=dtype, **knobs)
                gen = ref_codegen.generate(kern, cfg, "cpu", outdir=None, write=False)
                stem = "ref_omp_%s_%s_%s" % (name, dtype, cfg_name)
                src = os.path.join(GEN_DIR, stem + ".cpp")
                if not os.path.exists(src) or open(src).read() != gen.source:
                    with open(src, "w") as fh:
                        fh.write(gen.source)
                lib = os.path.join(REF_DIR, stem + ".so")
                if force or _stale(lib, [src]):
                    _compile_omp(cxx, src, lib, "-march=x86-64-v3")
                out[stem] = lib
                manifest[stem] = {"kernel": name, "dtype": dtype, "config": knobs,
                                  "abi": gen.abi_signature}
    with open(os.path.join(REF_DIR, "manifest.json"), "w") as fh:
        json.dump(manifest, fh, indent=1, sort_keys=True)
    return out


def _compile_omp(cxx: str, src: str, lib: str, march: str) -> None:
    # the reference's CPU flags (tilegen/verify.py:238-247, 304-305) with a given -march
    _run([cxx, "-std=c++17", "-shared", "-fPIC", "-o", lib, src, "-O3", march, "-fopenmp"])


def rebuild_ref_native(dest_dir: str) -> Optional[Dict[str, str]]:
    """Recompile the emitted reference OpenMP sources with -march=native into dest_dir
    (on the machine that will run them).  Returns {stem: path} or None if impossible."""
    cxx = shutil.which("g++") or shutil.which("c++")
    srcs = sorted(glob.glob(os.path.join(GEN_DIR, "ref_omp_*.cpp")))
    if cxx is None or not srcs:
        return None
    os.makedirs(dest_dir, exist_ok=True)
    out = {}
    for src in srcs:
        stem = os.path.basename(src)[:-4]
        lib = os.path.join(dest_dir, stem + ".so")
        try:
            _compile_omp(cxx, src, lib, "-march=native")
        except RuntimeError:
            return None
        out[stem] = lib
    return out


def main() -> int:
    print(build_oracle())
    for k, v in sorted(build_ref().items()):
        print(k, v)
    return 0


if __name__ == "__main__":
    sys.exit(main())
