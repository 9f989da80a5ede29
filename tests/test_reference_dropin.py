"""The b200 backend driven by the reference's own Python objects (CPU only).

With the reference tree present (``TILEGEN_REFERENCE_ROOT``, else ``reference`` beside
this repository), :func:`tilegen_b200.reference_patch.install` adds ``backend="b200"`` to
the reference's real modules.  Then the reference's ``standard_kernels()``
(tilegen/dsl.py:259-271) under its own ``Config`` (tilegen/codegen.py:61-87) go through
its real pass pipeline (tilegen/passes.py:450-470) inside its real ``generate()``
(tilegen/codegen.py:854-889), and the lowered kernel must give the same ``tg_sched`` as
this package's restatement of the lowering rules, for the seven schedules of the
reference's CUDA suite (tests/test_cuda_gpu.py:36-44) and the three of its
verify_all script (scripts/verify_all.py:26-30).  ``compile_generated`` must return
libtilegen_b200.so and leave the schedule for its ``launch_<name>`` entry points.
Skipped where the reference tree is absent (the GPU box).
"""

from __future__ import annotations

import os
import sys

import pytest

from tilegen_b200 import codegen as cg
from tilegen_b200 import lib
from tilegen_b200 import reference_patch

HERE = os.path.dirname(os.path.abspath(__file__))
REF_ROOT = os.environ.get("TILEGEN_REFERENCE_ROOT", os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference"))
HAVE_REF = os.path.exists(os.path.join(REF_ROOT, "tilegen", "passes.py"))

pytestmark = pytest.mark.skipif(not HAVE_REF, reason="reference tree not present")

KERNELS = ["spmv", "spmm", "sddmm", "fused_spmv_axpy", "axpy"]
SCHEDULES = [
    # tests/test_cuda_gpu.py:36-44
    dict(tile_size=32, threads_per_row=1, unroll=1, vector_width=1, block_size=128),
    dict(tile_size=32, threads_per_row=2, unroll=2, vector_width=1, block_size=128),
    dict(tile_size=64, threads_per_row=4, unroll=4, vector_width=2, block_size=256),
    dict(tile_size=128, threads_per_row=8, unroll=2, vector_width=2, block_size=512),
    dict(tile_size=32, threads_per_row=32, unroll=8, vector_width=2, block_size=512),
    dict(tile_size=1, threads_per_row=4, unroll=1, vector_width=1, block_size=128),
    dict(tile_size=256, threads_per_row=1, unroll=4, vector_width=1, block_size=256),
    # scripts/verify_all.py:26-30
    dict(tile_size=64, threads_per_row=1, unroll=4, vector_width=1, block_size=256),
]


@pytest.fixture(scope="module")
def ref():
    sys.path.insert(0, REF_ROOT)
    try:
        from tilegen import codegen as rc
        from tilegen import dsl as rd
        from tilegen import passes as rp
        from tilegen import verify as rv
    finally:
        sys.path.remove(REF_ROOT)
    reference_patch.install(rc, rv, rp)
    yield rc, rd, rp, rv
    reference_patch.uninstall()
    lib.set_schedule(lib.default_schedule())


@pytest.mark.parametrize("cfg", SCHEDULES, ids=lambda c: "T%d-TPR%d-U%d-V%d-B%d" % tuple(c.values()))
@pytest.mark.parametrize("name", KERNELS)
def test_reference_generate_lowers_to_the_same_schedule(ref, name, cfg):
    rc, rd, rp, rv = ref
    gen = rc.generate(rd.standard_kernels()[name], rc.Config(**cfg), "b200", write=False)
    assert isinstance(gen, cg.B200Kernel) and gen.kernel_name == name
    mine = cg.generate(name, cg.Config(**cfg))
    assert gen.sched.as_dict() == mine.sched.as_dict()
    assert gen.abi_signature == cg.STANDARD_KERNELS[name]
    # the reference pipeline's pass log travels with the descriptor
    assert any(e.get("pass") == "thread_mapping" if isinstance(e, dict) else "thread_mapping" in str(e)
               for e in gen.pass_log)


def test_reference_compile_generated_returns_the_library_and_sets_the_schedule(ref):
    rc, rd, rp, rv = ref
    cfg = rc.Config(**SCHEDULES[3])
    gen = rc.generate(rd.standard_kernels()["spmv"], cfg, "b200", write=False)
    path, log = rv.compile_generated(gen, "b200")
    assert os.path.samefile(path, lib.lib_path()) and "b200 prebuilt" in log
    assert lib.get_schedule().as_dict() == gen.sched.as_dict()


def test_reference_injected_bug_flag_reaches_the_schedule(ref):
    rc, rd, rp, rv = ref
    gen = rc.generate(rd.standard_kernels()["spmv"], rc.Config(inject_bug=True), "b200", write=False)
    assert gen.sched.flags & lib.TG_FLAG_INJECT_BUG


def test_other_backends_are_untouched(ref):
    rc, rd, rp, rv = ref
    gen = rc.generate(rd.standard_kernels()["spmv"], rc.Config(), "cpu", write=False)
    assert not isinstance(gen, cg.B200Kernel)
    assert "launch_spmv" in gen.source
