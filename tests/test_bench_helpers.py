"""bench.py's workload definitions: compulsory bytes (indptr + indices + values + dense
inputs + outputs, each once, at the BASELINE shapes), default schedules the library
accepts, row sharding."""

from __future__ import annotations

import importlib.util
import os

import numpy as np
import pytest

from tilegen_b200 import lib
from tilegen_b200.matrices import CSR

HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.fixture(scope="module")
def bench():
    spec = importlib.util.spec_from_file_location("bench", os.path.join(os.path.dirname(HERE), "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _toy():
    return CSR(np.array([0, 2, 3, 3, 6]), np.array([0, 3, 1, 0, 2, 3]), np.arange(1.0, 7.0), (4, 4), "toy")


def test_compulsory_bytes(bench):
    A = _toy()
    assert bench.matrix_bytes("c1", A) == 8 * 5 + 16 * 6 + 8 * 4 + 8 * 4
    assert bench.matrix_bytes("c5-spmm", A) == 8 * 5 + 12 * 6 + 4 * 4 * 128 + 4 * 4 * 128
    assert bench.matrix_bytes("c5-sddmm", A) == 8 * 5 + 12 * 6 + 4 * 4 * 64 * 2 + 4 * 6
    assert bench.spmv_bytes(8_000_000, 8_000_000, 256_000_000) == 4_288_000_008
    assert bench.matrix_flops("c5-spmm", A) == 2.0 * 6 * 128
    assert bench.matrix_bytes("blocked-spmm", A) == bench.matrix_bytes("c5-spmm", A)
    assert bench.matrix_kernel("blocked-spmm") == "spmm" and bench.matrix_kernel("c5-sddmm") == "sddmm"


def test_default_schedules_are_valid(bench):
    for wl, d in bench.SCHEDULES.items():
        bench.make_sched(d["split"], d["tpr"], d["unroll"], d["vec"], d["block"])  # raises on a rejected schedule
    assert set(bench.SCHEDULES) == set(bench.WORKLOADS)


def test_row_shard_rebases_indptr(bench):
    A = _toy()
    S = bench.row_shard(A, 1, 4)
    assert S.rows == 3 and S.cols == 4 and S.nnz == 4
    assert list(S.indptr) == [0, 1, 1, 4]
    assert list(S.indices) == [1, 0, 2, 3]


def test_inputs_are_seeded(bench):
    A = _toy()
    a = bench.matrix_inputs("c1", A)["x"]
    b = bench.matrix_inputs("c1", A)["x"]
    assert np.array_equal(a, b) and a.min() >= -1.0 and a.max() <= 1.0
    u = bench.matrix_inputs("c5-sddmm", A)
    assert u["U"].shape == (4, 64) and u["V"].shape == (4, 64) and u["U"].dtype == np.float32
