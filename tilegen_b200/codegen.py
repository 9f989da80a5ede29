"""The ``b200`` backend of TileGen's code generator.

TileGen turns a DSL kernel plus a :class:`Config` into schedule transforms with its pass
pipeline and then *emits source text* per backend (tilegen/codegen.py:854-889).  The
b200 backend does not emit source: the sm_100a kernels are written by hand and shipped
precompiled in libtilegen_b200.so, so ``generate(..., backend="b200")`` returns a
:class:`B200Kernel` descriptor -- the kernel id plus the template parameters read from
the lowered schedule -- and :func:`compile_generated` is a no-op that returns the
prebuilt library.

Two ways in:

* ``generate(kernel, config, "b200")`` with ``kernel`` a standard kernel name (or this
  package's own lowering), which applies the reference pipeline's lowering rules for the
  standard kernels (:func:`lower`, restating tilegen/passes.py:243-396);
* :func:`generate_from_lowered` with a kernel object that already went through the
  reference's ``passes.run_pipeline`` -- the schedule transforms (Tile, ThreadsPerRow,
  Unroll, Vectorize, Parallelize) are read from ``kernel.schedule`` exactly as the
  reference's ``_lowering`` does (tilegen/codegen.py:119-134).  This is the entry a
  maintainer calls from the reference's ``generate()`` for ``backend == "b200"``.
"""

from __future__ import annotations

import hashlib
import json
import os
from dataclasses import dataclass, field
from typing import Any, Dict, List, Optional, Sequence

from . import lib as _lib

__all__ = [
    "Config",
    "as_config",
    "Lowering",
    "B200Kernel",
    "STANDARD_KERNELS",
    "lower",
    "lowering_from_schedule",
    "generate",
    "generate_from_lowered",
    "compile_generated",
    "to_sched",
]

# The standard kernels of tilegen/dsl.py:259-271 and their launch ABIs
# (tilegen/codegen.py:_abi, 226-280).
STANDARD_KERNELS: Dict[str, str] = {
    "spmv": "void launch_spmv(const int64_t* indptr, const int64_t* indices, const double* data, "
            "const double* x, double* y, int64_t M, int64_t N, int64_t nnz)",
    "spmm": "void launch_spmm(const int64_t* indptr, const int64_t* indices, const double* data, "
            "const double* B, double* C, int64_t M, int64_t N, int64_t K, int64_t nnz)",
    "sddmm": "void launch_sddmm(const int64_t* indptr, const int64_t* indices, const double* data, "
             "const double* U, const double* V, double* C, int64_t M, int64_t N, int64_t K, int64_t nnz)",
    "fused_spmv_axpy": "void launch_fused_spmv_axpy(const int64_t* indptr, const int64_t* indices, "
                       "const double* data, const double* x, const double* w, double* z, double alpha, "
                       "double beta, int64_t M, int64_t N, int64_t nnz)",
    "axpy": "void launch_axpy(const double* x, const double* w, double* z, double alpha, double beta, "
            "int64_t M)",
}

# Kernels whose statements contain a rank-2 dense access (the only ones the reference's
# vectorize pass keeps Vectorize for, tilegen/passes.py:348-396).
_HAS_2D_DENSE = {"spmm", "sddmm"}
_SPLITS = {"rowwise": _lib.TG_SPLIT_ROWWISE, "merge": _lib.TG_SPLIT_MERGE, "auto": _lib.TG_SPLIT_AUTO,
           "stream": _lib.TG_SPLIT_STREAM, "block": _lib.TG_SPLIT_BLOCK}


@dataclass
class Config:
    """Schedule knobs (tilegen/codegen.py:61-87) plus the b200-only ones.

    ``split`` chooses the row mapping of the b200 kernels ("rowwise": the reference's
    T/TPR mapping; "merge": nnz-balanced chunks; "stream": the persistent TMA-fed SpMV,
    merge for SpMM/SDDMM; "block": SpMM over groups of 8 rows sharing a column list
    (block-structured matrices), merge for SpMV/SDDMM; "auto": merge), ``chunk_nnz`` the merge chunk size for
    SpMM/SDDMM, ``bounds_check`` a device-side CSR validation before the call."""

    tile_size: int = 32
    threads_per_row: int = 1
    unroll: int = 1
    vector_width: int = 1
    block_size: int = 256
    dtype: str = "f64"
    inject_bug: bool = False
    split: str = "rowwise"
    chunk_nnz: int = 0
    bounds_check: bool = False

    def to_dict(self) -> Dict[str, Any]:
        return {
            "tile_size": self.tile_size,
            "threads_per_row": self.threads_per_row,
            "unroll": self.unroll,
            "vector_width": self.vector_width,
            "block_size": self.block_size,
            "dtype": self.dtype,
            "inject_bug": self.inject_bug,
            "split": self.split,
            "chunk_nnz": self.chunk_nnz,
            "bounds_check": self.bounds_check,
        }

    def hash(self) -> str:
        """Same key as the reference for the shared knobs (tilegen/codegen.py:82-87);
        the b200 knobs are appended only when they differ from their defaults."""
        key = "%d|%d|%d|%d|%d|%s|%d" % (
            self.tile_size, self.threads_per_row, self.unroll, self.vector_width, self.block_size,
            self.dtype, int(self.inject_bug))
        if self.split != "rowwise" or self.chunk_nnz or self.bounds_check:
            key += "|%s|%d|%d" % (self.split, self.chunk_nnz, int(self.bounds_check))
        return hashlib.sha1(key.encode()).hexdigest()[:10]


@dataclass
class Lowering:
    """The launch decisions the kernels consume (tilegen/codegen.py:90-134) plus the
    b200 row split."""

    tile: int = 1
    threads_per_row: int = 1
    unroll: int = 1
    vector_width: int = 1
    block_size: int = 256
    parallel: bool = False
    split: str = "rowwise"
    chunk_nnz: int = 0

    def to_dict(self) -> Dict[str, Any]:
        return {
            "tile": self.tile,
            "threads_per_row": self.threads_per_row,
            "unroll": self.unroll,
            "vector_width": self.vector_width,
            "block_size": self.block_size,
            "parallel": self.parallel,
            "split": self.split,
            "chunk_nnz": self.chunk_nnz,
        }


def lower(kernel_name: str, config: Config, skip_passes: Sequence[str] = ()) -> Lowering:
    """The lowering the reference pipeline produces for a standard kernel.

    tiling (tilegen/passes.py:243-270): Tile(T) when T > 1;
    thread_mapping (:276-316): Parallelize(block=B), ThreadsPerRow(TPR) when TPR > 1;
    unroll (:322-342): Unroll(U) when U > 1;
    vectorize (:348-396): Vectorize(V) when V > 1.  The reference keeps Vectorize only
    for kernels with a rank-2 dense access (SpMM, SDDMM), because its emitted SpMV
    template has nothing to vectorise; the b200 SpMV template reads the CSR stream
    (indices, values) with V-wide vector loads, so V is kept for every kernel.
    A skipped pass leaves its knob at the Lowering default, as in the reference.
    """
    if kernel_name not in STANDARD_KERNELS:
        raise ValueError("unknown kernel %r" % kernel_name)
    skip = set(skip_passes)
    low = Lowering(split=config.split, chunk_nnz=config.chunk_nnz)
    if "tiling" not in skip and config.tile_size > 1:
        low.tile = config.tile_size
    if "thread_mapping" not in skip:
        low.parallel = True
        low.block_size = config.block_size or 256
        if config.threads_per_row > 1:
            low.threads_per_row = config.threads_per_row
    if "unroll" not in skip and config.unroll > 1:
        low.unroll = config.unroll
    if "vectorize" not in skip and config.vector_width > 1:
        low.vector_width = config.vector_width
    return low


def lowering_from_schedule(schedule, split: str = "rowwise", chunk_nnz: int = 0) -> Lowering:
    """Read a reference schedule (an iterable of Tile / ThreadsPerRow / Unroll /
    Vectorize / Parallelize transforms) the way tilegen/codegen.py:119-134 does.  The
    transforms are matched by class name, so the reference's IR classes work without
    importing them."""
    low = Lowering(split=split, chunk_nnz=chunk_nnz)
    for t in schedule:
        kind = type(t).__name__
        if kind == "Tile":
            low.tile = int(t.size)
        elif kind == "ThreadsPerRow":
            low.threads_per_row = int(t.k)
        elif kind == "Unroll":
            low.unroll = int(t.factor)
        elif kind == "Vectorize":
            low.vector_width = int(t.width)
        elif kind == "Parallelize":
            low.parallel = True
            if getattr(t, "block_size", 0):
                low.block_size = int(t.block_size)
    return low


def to_sched(low: Lowering, config: Optional[Config] = None) -> _lib.TgSched:
    """Lowering -> the C ABI's tg_sched (one field per template parameter)."""
    s = _lib.TgSched()
    s.tile = max(1, int(low.tile))
    s.threads_per_row = int(low.threads_per_row)
    s.unroll = int(low.unroll)
    s.vector_width = int(low.vector_width)
    s.block_size = int(low.block_size)
    if low.split not in _SPLITS:
        raise ValueError("split must be one of %s (got %r)" % (sorted(_SPLITS), low.split))
    s.split = _SPLITS[low.split]
    s.chunk_nnz = int(low.chunk_nnz)
    flags = 0
    if config is not None and config.inject_bug:
        flags |= _lib.TG_FLAG_INJECT_BUG
    if config is not None and config.bounds_check:
        flags |= _lib.TG_FLAG_BOUNDS_CHECK
    s.flags = flags
    return s


@dataclass
class B200Kernel:
    """What ``generate(..., "b200")`` returns: the descriptor of a prebuilt kernel
    instance (kernel id + template parameters), in place of generated source."""

    kernel_name: str
    config: Config
    lowering: Lowering
    abi_signature: str
    pass_log: List[Dict[str, Any]] = field(default_factory=list)
    backend: str = "b200"

    @property
    def sched(self) -> _lib.TgSched:
        return to_sched(self.lowering, self.config)

    @property
    def source(self) -> str:
        return json.dumps({"backend": "b200", "kernel": self.kernel_name, "config": self.config.to_dict(),
                           "lowering": self.lowering.to_dict(), "abi": self.abi_signature}, sort_keys=True)

    @property
    def filename(self) -> str:
        digest = hashlib.sha1(self.source.encode()).hexdigest()[:8]
        return "%s_%s_%s.b200.json" % (self.kernel_name, self.config.hash(), digest)

    def write(self, outdir: str = "build/generated") -> str:
        os.makedirs(outdir, exist_ok=True)
        path = os.path.join(outdir, self.filename)
        with open(path, "w") as fh:
            fh.write(self.source)
        return path


def generate(kernel, config: Config, backend: str = "b200", outdir: Optional[str] = None, write: bool = False,
             skip_passes: Sequence[str] = ()) -> B200Kernel:
    """``tilegen.codegen.generate`` for the b200 backend.  ``kernel`` is a standard
    kernel name or a kernel object with a ``name`` (its schedule is lowered from
    ``config`` with the reference pipeline's rules)."""
    if backend != "b200":
        raise ValueError("this package implements only the 'b200' backend (got %r)" % backend)
    name = kernel if isinstance(kernel, str) else getattr(kernel, "name")
    low = lower(name, config, skip_passes)
    log = [{"pass": p, "action": "lowered for b200"} for p in
           ("tiling", "thread_mapping", "unroll", "vectorize") if p not in set(skip_passes)]
    gen = B200Kernel(name, config, low, STANDARD_KERNELS[name], pass_log=log)
    if write and outdir:
        gen.write(outdir)
    return gen


def as_config(config) -> Config:
    """This package's Config from any object with the reference Config's fields
    (tilegen/codegen.py:61-69: tile_size, threads_per_row, unroll, vector_width,
    block_size, dtype, inject_bug); the b200-only knobs take their defaults unless the
    object has them."""
    if isinstance(config, Config):
        return config
    d = Config()
    kw = {f: getattr(config, f, getattr(d, f)) for f in
          ("tile_size", "threads_per_row", "unroll", "vector_width", "block_size", "dtype", "inject_bug", "split",
           "chunk_nnz", "bounds_check")}
    return Config(**kw)


def generate_from_lowered(optimized_kernel, config) -> B200Kernel:
    """Build the descriptor from a kernel the reference's pass pipeline already lowered
    (reads ``optimized_kernel.schedule`` and ``.pass_log``).  ``config`` may be the
    reference's own Config object."""
    config = as_config(config)
    name = optimized_kernel.name
    if name not in STANDARD_KERNELS:
        raise NotImplementedError("the b200 backend has kernels for %s (got %r)" % (sorted(STANDARD_KERNELS), name))
    low = lowering_from_schedule(optimized_kernel.schedule, config.split, config.chunk_nnz)
    if name not in _HAS_2D_DENSE and low.vector_width == 1:
        # the reference's vectorize pass dropped V for a kernel without a rank-2 dense
        # access; the b200 template vectorises the CSR stream, so take V from the config
        low.vector_width = max(1, int(config.vector_width))
    return B200Kernel(name, config, low, STANDARD_KERNELS[name],
                      pass_log=list(getattr(optimized_kernel, "pass_log", []) or []))


def compile_generated(gen: B200Kernel, backend: str = "b200", workdir: Optional[str] = None, verbose: bool = False):
    """No compilation for b200: returns (path of the prebuilt library, log).  Raises
    LibraryError if the library is missing (no fallback)."""
    _lib.load()
    return _lib.lib_path(), "b200 prebuilt %s (%s) kernel=%s sched=%s" % (
        os.path.basename(_lib.lib_path()), _lib.version(), gen.kernel_name, gen.sched.as_dict())
