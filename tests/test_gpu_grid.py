"""The reference's full differential grid on the GPU.

Mirrors scripts/verify_all.py:24-30 of the reference: every corpus class
(tilegen/matrices.py:164-178, generated bit for bit by tilegen_b200.matrices) x the five
standard kernels x the script's three configs, plus one injected-bug SpMV per class that
the harness must catch.  Each result is checked two ways: by ``verify`` (the reference's
SciPy float64 expectation and acceptance rule, tilegen/verify.py:350-371, 510-514) and
against the CPU oracle on the same inputs (max relative error <= 1e-9, with the relative
error floored at 1e-3 of the largest reference magnitude).  The whole grid runs once with
the reference's rowwise mapping and once with the merge split.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import oracle as O
from tilegen_b200 import codegen as cg
from tilegen_b200 import lib
from tilegen_b200 import matrices as M
from tilegen_b200.verify import inputs_for, run_kernel, verify

pytestmark = pytest.mark.gpu

KERNELS = ["spmv", "spmm", "sddmm", "fused_spmv_axpy", "axpy"]

# scripts/verify_all.py:26-30
CONFIGS = [
    dict(tile_size=32, threads_per_row=1, unroll=1, vector_width=1, block_size=128),
    dict(tile_size=64, threads_per_row=1, unroll=4, vector_width=1, block_size=256),
    dict(tile_size=128, threads_per_row=8, unroll=2, vector_width=2, block_size=512),
]
CONFIG_IDS = ["T32-U1-B128", "T64-U4-B256", "T128-TPR8-U2-V2-B512"]
SPLITS = ["rowwise", "merge"]

_matrices = {}


def _matrix(cls):
    if cls not in _matrices:
        _matrices[cls] = M.make_matrix(cls)
    return _matrices[cls]


def _rel(out, ref):
    out, ref = np.asarray(out, np.float64).ravel(), np.asarray(ref, np.float64).ravel()
    if ref.size == 0:
        return 0.0
    floor = 1e-3 * max(float(np.abs(ref).max()), 1e-300)
    return float((np.abs(out - ref) / np.maximum(np.abs(ref), floor)).max())


def _oracle(kernel, A, data):
    x, w, B, U, V, a, b = data
    if kernel == "spmv":
        return O.spmv(A, x)
    if kernel == "spmm":
        return O.spmm(A, B)
    if kernel == "sddmm":
        return O.sddmm(A, U, V)
    if kernel == "fused_spmv_axpy":
        return O.fused_spmv_axpy(A, x, w, a, b)
    return O.axpy(x, w, a, b)


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    lib.load()
    yield
    _matrices.clear()


@pytest.mark.parametrize("split", SPLITS)
@pytest.mark.parametrize("cfg", CONFIGS, ids=CONFIG_IDS)
@pytest.mark.parametrize("kernel", KERNELS)
@pytest.mark.parametrize("cls", M.corpus_classes())
def test_grid(cls, kernel, cfg, split):
    A = _matrix(cls)
    config = cg.Config(split=split, **cfg)
    res = verify(kernel, config, A, K=8)
    assert res.ok, res.to_dict()
    # the same call again, compared with the oracle instead of SciPy
    data = inputs_for(kernel, A, 8, 7)
    out = run_kernel(cg.generate(kernel, config), A, data, K=8)
    assert _rel(out, _oracle(kernel, A, data)) <= 1e-9


@pytest.mark.parametrize("split", SPLITS)
@pytest.mark.parametrize("cls", M.corpus_classes())
def test_grid_injected_bug_is_caught(cls, split):
    """scripts/verify_all.py:57-60: the deliberately buggy SpMV must fail."""
    A = _matrix(cls)
    res = verify("spmv", cg.Config(tile_size=32, threads_per_row=1, unroll=1, inject_bug=True, split=split), A)
    assert not res.ok and res.max_abs_err > res.tolerance, res.to_dict()
