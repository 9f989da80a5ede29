"""The ``b200`` backend added to TileGen's own modules at run time.

TileGen reaches a kernel through ``tilegen.codegen.generate(kernel, config, backend)``
(tilegen/codegen.py:854-889), ``tilegen.verify.compile_generated`` (tilegen/verify.py:
264-312) and ``tilegen.verify.run_kernel`` (tilegen/verify.py:414-451); ``verify()``
looks all three up when it runs (tilegen/verify.py:455-530).  :func:`install` wraps them
so that ``backend="b200"``

* runs the reference's own pass pipeline (``tilegen.passes.run_pipeline``,
  tilegen/passes.py:450-470) on the kernel and hands the lowered kernel to
  :func:`tilegen_b200.codegen.generate_from_lowered` (a descriptor of the prebuilt
  kernel instance instead of emitted source);
* "compiles" by returning the path of libtilegen_b200.so and setting the process-global
  schedule its ``launch_<name>`` entry points read (``tg_set_schedule``);
* runs the kernel exactly as the reference runs a generated CUDA object: buffers
  mirrored to the device by the reference's ``_CudaBuffers``, the ``launch_<name>`` call
  with the reference's ctypes signatures, a device synchronize, the copy back.

Every other backend goes to the reference's original functions unchanged.  These are
the same three edits a maintainer would make in the reference's source (one ``if
backend == "b200"`` branch in each function); :func:`install` applies them without
editing the tree, and :func:`uninstall` removes them.
"""

from __future__ import annotations

from typing import Any, Dict, Optional

_saved: Optional[Dict[str, Any]] = None


def install(codegen_mod, verify_mod, passes_mod) -> None:
    """Add the b200 backend to the given ``tilegen.codegen``, ``tilegen.verify`` and
    ``tilegen.passes`` modules (idempotent)."""
    global _saved
    if _saved is not None:
        return
    from . import codegen as b200_codegen
    from . import lib as tgl

    orig_generate = codegen_mod.generate
    orig_compile = verify_mod.compile_generated
    orig_run = verify_mod.run_kernel

    def generate(kernel, config, backend="cpu", outdir="build/generated", write=True, skip_passes=()):
        if backend != "b200":
            return orig_generate(kernel, config, backend, outdir=outdir, write=write, skip_passes=skip_passes)
        optimized = passes_mod.run_pipeline(kernel, config, backend=backend, skip=skip_passes)
        gen = b200_codegen.generate_from_lowered(optimized, config)
        if write and outdir:
            gen.write(outdir)
        return gen

    def compile_generated(gen, backend="cpu", workdir="build/generated", verbose=False):
        if backend != "b200":
            return orig_compile(gen, backend, workdir, verbose)
        path, log = b200_codegen.compile_generated(gen)
        tgl.set_schedule(gen.sched)  # read by launch_<name> on the next call
        return path, log

    def run_kernel(lib_path, kernel_name, A, data, K=8, backend="cpu"):
        # the library's launchers take device pointers, as a generated CUDA object does
        return orig_run(lib_path, kernel_name, A, data, K, backend="cuda" if backend == "b200" else backend)

    _saved = {"generate": orig_generate, "compile_generated": orig_compile, "run_kernel": orig_run,
              "mods": (codegen_mod, verify_mod)}
    codegen_mod.generate = generate
    verify_mod.compile_generated = compile_generated
    verify_mod.run_kernel = run_kernel


def uninstall() -> None:
    """Restore the reference's original functions."""
    global _saved
    if _saved is None:
        return
    codegen_mod, verify_mod = _saved["mods"]
    codegen_mod.generate = _saved["generate"]
    verify_mod.compile_generated = _saved["compile_generated"]
    verify_mod.run_kernel = _saved["run_kernel"]
    _saved = None
