"""Record how the reference's own ``verify()`` drives a CUDA kernel library, for replay
on the GPU box (where the reference's Python is not available).

With the b200 backend installed into the reference's modules
(tilegen_b200.reference_patch.install), this runs the reference's
``tilegen.verify.verify(kernel, Config(...), <257x257 edge matrix>, backend="b200")``
(tilegen/verify.py:455-530) for every standard kernel and two schedules, with two
stand-ins that only record: the CUDA runtime the reference loads for its device buffers
(``_cuda_runtime``, tilegen/verify.py:52-101; host memory plays device memory) and the
``ctypes.CDLL`` it opens libtilegen_b200.so with (tilegen/verify.py:422-424).  Each call is
written to ``ref_run_kernel_calls.json``: the schedule that compile_generated left, every
cudaMalloc, cudaMemcpy (a host-to-device copy names the golden array whose bytes it
copies), cudaDeviceSynchronize and cudaFree, and the ``launch_<name>`` call with the ctypes
types the reference set and its arguments (device buffers by index, scalars by value).

Run in a checkout with the reference tree (``TILEGEN_REFERENCE_ROOT``, else ``reference``
beside this repository):  python tests/golden/make_run_kernel_transcript.py
"""

from __future__ import annotations

import ctypes
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
REF_ROOT = os.environ.get("TILEGEN_REFERENCE_ROOT", os.path.join(os.path.dirname(REPO), "reference"))

KERNELS = ["spmv", "spmm", "sddmm", "fused_spmv_axpy", "axpy"]
SCHEDULES = {"T32-TPR1-U1-V1-B128": dict(tile_size=32, threads_per_row=1, unroll=1, vector_width=1, block_size=128),
             "T128-TPR8-U2-V2-B512": dict(tile_size=128, threads_per_row=8, unroll=2, vector_width=2,
                                          block_size=512)}


class _Runtime:
    """Records the CUDA runtime calls of the reference's _CudaBuffers."""

    def __init__(self, golden):
        self.events = []
        self.golden = golden  # name -> bytes
        self.bufs = {}  # stand-in device address -> (index, buffer)

    def _name(self, addr, n):
        data = ctypes.string_at(addr, n)
        for name, b in self.golden.items():
            if b == data:
                return name
        return "zeros" if data == bytes(n) else "unknown"

    def cudaMalloc(self, pptr, size):
        n = int(size.value)
        buf = ctypes.create_string_buffer(max(n, 1))
        self.bufs[ctypes.addressof(buf)] = (len(self.bufs), buf)
        pptr._obj.value = ctypes.addressof(buf)
        self.events.append({"op": "malloc", "buf": len(self.bufs) - 1, "bytes": n})
        return 0

    def cudaMemcpy(self, dst, src, size, kind):
        n = int(size.value)
        if int(kind) == 1:  # cudaMemcpyHostToDevice
            self.events.append({"op": "h2d", "buf": self.bufs[dst.value][0], "bytes": n,
                                "src": self._name(src.value, n)})
        else:
            self.events.append({"op": "d2h", "buf": self.bufs[src.value][0], "bytes": n})
        ctypes.memmove(dst.value, src.value, n)
        return 0

    def cudaDeviceSynchronize(self):
        self.events.append({"op": "sync"})
        return 0

    def cudaFree(self, ptr):
        self.events.append({"op": "free", "buf": self.bufs[ptr.value][0]})
        return 0

    def cudaGetErrorString(self, code):
        return b"recorded"


class _Launch:
    def __init__(self, rt, symbol):
        self.rt, self.symbol, self.argtypes, self.restype = rt, symbol, None, None

    def __call__(self, *args):
        out = []
        for a in args:
            addr = ctypes.cast(a, ctypes.c_void_p).value if isinstance(a, ctypes._Pointer) else None
            if addr is not None and addr in self.rt.bufs:
                out.append({"buf": self.rt.bufs[addr][0]})
            else:
                out.append({"scalar": a})
        self.rt.events.append({"op": "launch", "symbol": self.symbol,
                               "argtypes": [t.__name__ for t in self.argtypes], "args": out})


class _Library:
    def __init__(self, rt):
        self.rt = rt

    def __getattr__(self, name):
        if name.startswith("launch_"):
            return _Launch(self.rt, name)
        raise AttributeError(name)


def main() -> int:
    sys.path.insert(0, REPO)
    sys.path.insert(0, REF_ROOT)
    import scipy.sparse as sp

    from tilegen import codegen as rc, passes as rp, verify as rv  # noqa: E402  (reference tree)

    from tilegen_b200 import lib, reference_patch  # noqa: E402

    lib.load()  # before CDLL is replaced below
    z = np.load(os.path.join(HERE, "edge257.npz"))
    A = sp.csr_matrix((z["data"], z["indices"], z["indptr"]), shape=tuple(int(s) for s in z["shape"]))
    golden = {k: np.ascontiguousarray(z[k]).tobytes() for k in ("indptr", "indices", "data", "x", "w", "B", "U", "V")}
    real_cdll, real_rt = rv.ctypes.CDLL, rv._cuda_runtime
    cases = []
    reference_patch.install(rc, rv, rp)
    try:
        for sname, knobs in SCHEDULES.items():
            for kernel in KERNELS:
                rt = _Runtime(golden)
                rv._cuda_runtime = lambda rt=rt: rt
                rv.ctypes.CDLL = (lambda path, *a, rt=rt, **kw: _Library(rt) if os.path.basename(str(path)) ==
                                  "libtilegen_b200.so" else real_cdll(path, *a, **kw))
                rv.verify(kernel, rc.Config(**knobs), A, backend="b200", K=int(z["K"]))
                rv.ctypes.CDLL = real_cdll
                cases.append({"kernel": kernel, "schedule_name": sname, "config": knobs,
                              "sched": lib.get_schedule().as_dict(), "events": rt.events})
    finally:
        rv.ctypes.CDLL, rv._cuda_runtime = real_cdll, real_rt
        reference_patch.uninstall()
        lib.set_schedule(lib.default_schedule())
    with open(os.path.join(HERE, "ref_run_kernel_calls.json"), "w") as fh:
        json.dump({"matrix": "edge257 (the reference suite's 257x257 matrix, tests/test_cuda_gpu.py:53-76)",
                   "K": int(z["K"]), "cases": cases}, fh, indent=1)
    print("wrote %d cases" % len(cases))
    return 0


if __name__ == "__main__":
    sys.exit(main())
