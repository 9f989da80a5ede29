"""Build libtilegen_b200.so in-tree with nvcc for sm_100a.

Every ``csrc/*.cu`` translation unit is compiled to an object under
``tilegen_b200/_build/`` (in parallel, only when the source or a header changed) and
the objects are linked into ``tilegen_b200/libtilegen_b200.so``.  The CUDA runtime is
linked statically, so the library needs only the driver at run time.

Usage: ``python -m tilegen_b200.build [--force] [--jobs N]``.
"""

from __future__ import annotations

import argparse
import glob
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from typing import List

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
REPO_DIR = os.path.dirname(PKG_DIR)
CSRC = os.path.join(PKG_DIR, "csrc")
BUILD = os.path.join(PKG_DIR, "_build")
LIB_NAME = "libtilegen_b200.so"
LIB_PATH = os.path.join(PKG_DIR, LIB_NAME)

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "-Xcompiler",
    "-fPIC,-O3,-fvisibility=hidden",
    "-Xptxas",
    "-O3",
    "-I" + os.path.join(REPO_DIR, "include"),
]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: set NVCC or put /usr/local/cuda/bin on PATH")


def _headers() -> List[str]:
    return glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(REPO_DIR, "include", "*.h"))


def _stale(target: str, deps: List[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _compile(nvcc: str, src: str, obj: str, verbose: bool) -> None:
    cmd = [nvcc, *ARCH_FLAGS, *NVCC_FLAGS, "-c", src, "-o", obj]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError("nvcc failed for %s:\n%s%s" % (os.path.basename(src), res.stdout, res.stderr))


def build(force: bool = False, jobs: int = 0, verbose: bool = False) -> str:
    """Compile (incrementally) and link the library; return its path."""
    nvcc = nvcc_path()
    os.makedirs(BUILD, exist_ok=True)
    sources = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    headers = _headers()
    todo = []
    objs = []
    for src in sources:
        obj = os.path.join(BUILD, os.path.basename(src)[:-3] + ".o")
        objs.append(obj)
        if force or _stale(obj, [src, *headers]):
            todo.append((src, obj))
    if todo:
        jobs = jobs or min(len(todo), os.cpu_count() or 4)
        with ThreadPoolExecutor(max_workers=jobs) as ex:
            for fut in [ex.submit(_compile, nvcc, s, o, verbose) for s, o in todo]:
                fut.result()
    if force or todo or _stale(LIB_PATH, objs):
        cmd = [nvcc, *ARCH_FLAGS, "-shared", "-cudart", "static", "-o", LIB_PATH, *objs]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError("link failed:\n%s%s" % (res.stdout, res.stderr))
    build_cli(nvcc, force)
    build_probe(nvcc, force)
    return LIB_PATH


PROBE_SRC = os.path.join(PKG_DIR, "bench_probe", "tg_gather_probe.cu")
PROBE_PATH = os.path.join(PKG_DIR, "bench_probe", "libtg_gather_probe.so")


def build_probe(nvcc: str, force: bool = False) -> str:
    """The benchmark's gather-floor probe, a library of its own (not part of
    libtilegen_b200.so)."""
    if force or _stale(PROBE_PATH, [PROBE_SRC, *_headers()]):
        cmd = [nvcc, *ARCH_FLAGS, *NVCC_FLAGS, "-shared", "-cudart", "static", "-o", PROBE_PATH, PROBE_SRC]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError("gather probe build failed:\n%s%s" % (res.stdout, res.stderr))
    return PROBE_PATH


CLI_SRC = os.path.join(PKG_DIR, "cli", "tilegen_b200_bench.cpp")
CLI_PATH = os.path.join(PKG_DIR, "tilegen_b200_bench")


def build_cli(nvcc: str, force: bool = False) -> str:
    """The C++ bench harness (the b200 counterpart of the reference's tilegen_bench): host
    code only; it dlopen()s the library at run time."""
    if force or _stale(CLI_PATH, [CLI_SRC, *_headers()]):
        cmd = [nvcc, "-O2", "-std=c++17", "-o", CLI_PATH, CLI_SRC, "-ldl"]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError("bench harness build failed:\n%s%s" % (res.stdout, res.stderr))
    return CLI_PATH


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=0)
    ap.add_argument("-v", "--verbose", action="store_true")
    args = ap.parse_args(argv)
    path = build(force=args.force, jobs=args.jobs, verbose=args.verbose)
    print(path)
    return 0


if __name__ == "__main__":
    sys.exit(main())
