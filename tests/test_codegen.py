"""The b200 backend's Config -> Lowering -> tg_sched mapping (tilegen/passes.py rules)."""

from __future__ import annotations

import hashlib
from dataclasses import dataclass

import pytest

from tilegen_b200 import codegen as cg
from tilegen_b200 import lib


def test_config_hash_matches_reference_formula_for_shared_knobs():
    c = cg.Config(tile_size=64, threads_per_row=8, unroll=2, vector_width=2, block_size=128)
    key = "%d|%d|%d|%d|%d|%s|%d" % (64, 8, 2, 2, 128, "f64", 0)  # tilegen/codegen.py:82-87
    assert c.hash() == hashlib.sha1(key.encode()).hexdigest()[:10]
    assert cg.Config(split="merge").hash() != cg.Config().hash()


def test_lowering_rules_for_standard_kernels():
    cfg = cg.Config(tile_size=128, threads_per_row=8, unroll=4, vector_width=2, block_size=512)
    spmv = cg.lower("spmv", cfg)
    # V is kept for SpMV too: the b200 template loads the CSR stream V-wide (the
    # reference drops it there because its SpMV template has nothing to vectorise)
    assert (spmv.tile, spmv.threads_per_row, spmv.unroll, spmv.vector_width, spmv.block_size) == (128, 8, 4, 2, 512)
    spmm = cg.lower("spmm", cfg)
    assert spmm.vector_width == 2  # rank-2 dense access keeps Vectorize
    t1 = cg.lower("spmv", cg.Config(tile_size=1, threads_per_row=1))
    assert t1.tile == 1 and t1.threads_per_row == 1


def test_skipped_passes_leave_defaults():
    cfg = cg.Config(tile_size=128, threads_per_row=8, unroll=4, vector_width=2, block_size=512)
    low = cg.lower("spmm", cfg, skip_passes=("tiling", "unroll", "vectorize", "thread_mapping"))
    assert (low.tile, low.threads_per_row, low.unroll, low.vector_width, low.block_size) == (1, 1, 1, 1, 256)
    assert not low.parallel


def test_lowering_from_reference_schedule_objects():
    """Transforms are matched by class name like tilegen/codegen.py:119-134."""

    @dataclass
    class Tile:
        size: int

    @dataclass
    class ThreadsPerRow:
        k: int

    @dataclass
    class Unroll:
        factor: int

    @dataclass
    class Vectorize:
        width: int

    @dataclass
    class Parallelize:
        block_size: int

    @dataclass
    class Kernel:
        name: str
        schedule: list
        pass_log: list

    k = Kernel("spmv", [Tile(64), Parallelize(256), ThreadsPerRow(4), Unroll(2), Vectorize(2)], [{"pass": "x"}])
    g = cg.generate_from_lowered(k, cg.Config())
    assert (g.lowering.tile, g.lowering.threads_per_row, g.lowering.unroll, g.lowering.block_size) == (64, 4, 2, 256)
    assert g.lowering.vector_width == 2
    assert g.pass_log == [{"pass": "x"}]
    # the reference pipeline drops Vectorize for SpMV: V then comes from the config
    k2 = Kernel("spmv", [Tile(64), Parallelize(256), ThreadsPerRow(4), Unroll(2)], [])
    assert cg.generate_from_lowered(k2, cg.Config(vector_width=4)).lowering.vector_width == 4
    assert cg.generate_from_lowered(k2, cg.Config()).lowering.vector_width == 1
    with pytest.raises(NotImplementedError):
        cg.generate_from_lowered(Kernel("mystery", [], []), cg.Config())


def test_to_sched_flags_and_split():
    g = cg.generate("spmv", cg.Config(inject_bug=True, split="merge", bounds_check=True))
    s = g.sched
    assert s.split == lib.TG_SPLIT_MERGE
    assert s.flags & lib.TG_FLAG_INJECT_BUG and s.flags & lib.TG_FLAG_BOUNDS_CHECK
    lib.validate_schedule(s)
    with pytest.raises(ValueError):
        cg.to_sched(cg.Lowering(split="diagonal"))


def test_generate_descriptor_and_compile_is_prebuilt(tmp_path):
    g = cg.generate("sddmm", cg.Config(vector_width=4), outdir=str(tmp_path), write=True)
    assert g.backend == "b200" and g.abi_signature.startswith("void launch_sddmm(")
    assert (tmp_path / g.filename).exists()
    path, log = cg.compile_generated(g)
    assert path.endswith("libtilegen_b200.so") and "b200 prebuilt" in log
    with pytest.raises(ValueError):
        cg.generate("spmv", cg.Config(), backend="cuda")
