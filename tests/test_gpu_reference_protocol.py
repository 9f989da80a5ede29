"""libtilegen_b200.so driven exactly the way the reference's own verify() drives a CUDA
kernel library.

tests/golden/ref_run_kernel_calls.json was recorded from the reference's
``tilegen.verify.verify(..., backend="b200")`` (tilegen/verify.py:455-530, with the b200
backend installed by tilegen_b200.reference_patch) by make_run_kernel_transcript.py: the
schedule compile_generated set, the reference's _CudaBuffers calls (cudaMalloc, cudaMemcpy
of named host arrays, cudaDeviceSynchronize, cudaFree; tilegen/verify.py:103-163) and the
``launch_<name>`` call with the ctypes argument types the reference assigned
(tilegen/verify.py:166-173, 422-424).  Here the same calls run against the real CUDA
runtime and the real library, on the reference suite's 257x257 edge matrix, and the
copied-back output is checked against the reference's SciPy float64 output under the
reference tolerance and the 1e-9 relative bar.
"""

from __future__ import annotations

import ctypes
import ctypes.util
import glob
import json
import os

import numpy as np
import pytest

from tilegen_b200 import lib
from tilegen_b200.verify import tolerance

from conftest import GOLDEN, load_npz

pytestmark = pytest.mark.gpu

with open(os.path.join(GOLDEN, "ref_run_kernel_calls.json")) as _fh:
    TRANSCRIPT = json.load(_fh)

CTYPES = {"c_long": ctypes.c_long, "c_longlong": ctypes.c_longlong, "c_double": ctypes.c_double,
          "LP_c_long": ctypes.POINTER(ctypes.c_long), "LP_c_longlong": ctypes.POINTER(ctypes.c_longlong),
          "LP_c_double": ctypes.POINTER(ctypes.c_double)}


def _cudart():
    """The CUDA runtime, found the way the reference looks for it (tilegen/verify.py:52-70)."""
    cands = [ctypes.util.find_library("cudart")] + sorted(glob.glob("/usr/local/cuda*/lib64/libcudart.so*"),
                                                          reverse=True)
    for c in cands:
        if not c:
            continue
        try:
            rt = ctypes.CDLL(c)
        except OSError:
            continue
        rt.cudaMalloc.argtypes = [ctypes.POINTER(ctypes.c_void_p), ctypes.c_size_t]
        rt.cudaMemcpy.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int]
        rt.cudaFree.argtypes = [ctypes.c_void_p]
        return rt
    pytest.fail("no CUDA runtime library found")


@pytest.mark.parametrize("case", TRANSCRIPT["cases"], ids=lambda c: "%s-%s" % (c["kernel"], c["schedule_name"]))
def test_reference_call_sequence_replayed(case):
    z = load_npz("edge257.npz")
    rt = _cudart()
    s = lib.TgSched(**case["sched"])
    lib.set_schedule(s)  # what the reference's compile_generated left for the launchers
    L = ctypes.CDLL(lib.lib_path())  # opened as the reference opens a kernel library
    bufs = {}
    host = {}
    out = None
    try:
        for e in case["events"]:
            op = e["op"]
            if op == "malloc":
                p = ctypes.c_void_p()
                assert rt.cudaMalloc(ctypes.byref(p), max(1, e["bytes"])) == 0
                bufs[e["buf"]] = (p, e["bytes"])
            elif op == "h2d":
                src = np.zeros(e["bytes"], np.uint8) if e["src"] == "zeros" else np.ascontiguousarray(z[e["src"]])
                assert src.nbytes == e["bytes"], (e, src.nbytes)
                host[e["buf"]] = src
                assert rt.cudaMemcpy(bufs[e["buf"]][0], src.ctypes.data, e["bytes"], 1) == 0
            elif op == "launch":
                fn = getattr(L, e["symbol"])
                fn.argtypes = [CTYPES[t] for t in e["argtypes"]]
                fn.restype = None
                args = [ctypes.cast(bufs[a["buf"]][0], t) if "buf" in a else a["scalar"]
                        for a, t in zip(e["args"], fn.argtypes)]
                fn(*args)
                assert lib.load().tg_last_status() == lib.TG_OK, lib.last_error()
            elif op == "sync":
                assert rt.cudaDeviceSynchronize() == 0
            elif op == "d2h":
                out = np.empty(e["bytes"] // 8, np.float64)
                assert rt.cudaMemcpy(out.ctypes.data, bufs[e["buf"]][0], e["bytes"], 2) == 0
            elif op == "free":
                assert rt.cudaFree(bufs.pop(e["buf"])[0]) == 0
    finally:
        for p, _ in bufs.values():
            rt.cudaFree(p)
        lib.set_schedule(lib.default_schedule())
    ref = np.asarray(z["ref_" + case["kernel"]], np.float64).ravel()
    assert out is not None and out.size == ref.size
    from tilegen_b200.matrices import CSR

    A = CSR(z["indptr"], z["indices"], z["data"], tuple(int(v) for v in z["shape"]), "edge257")
    d = float(np.abs(out - ref).max())
    assert d <= tolerance(A, ref), d
    floor = 1e-3 * float(np.abs(ref).max())
    assert float((np.abs(out - ref) / np.maximum(np.abs(ref), floor)).max()) <= 1e-9
