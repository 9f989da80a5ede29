"""The C++ bench harness (tilegen_b200_bench): command line and JSON line of the
reference's tilegen_bench (cpp/src/harness.cpp:117-268) on TGM1 files."""

from __future__ import annotations

import json
import os
import subprocess

import pytest

from tilegen_b200 import matrices as M

HERE = os.path.dirname(os.path.abspath(__file__))
CLI = os.path.join(os.path.dirname(HERE), "tilegen_b200", "tilegen_b200_bench")


def _run(*args):
    return subprocess.run([CLI, *args], capture_output=True, text=True, timeout=300)


def test_cli_usage_and_bad_input(tmp_path):
    assert os.path.exists(CLI), "build() makes the harness next to the library"
    r = _run()
    assert r.returncode == 2 and "usage" in r.stderr
    bad = tmp_path / "bad.bin"
    bad.write_bytes(b"NOPE" + b"\0" * 24)
    r = _run("--kernel", "spmv", "--matrix", str(bad))
    assert r.returncode == 2 and "not a TGM1 file" in r.stderr
    good = tmp_path / "m.bin"
    M.write_tgm1(str(good), M.edge_matrix())
    r = _run("--kernel", "spmv", "--matrix", str(good), "--split", "diagonal")
    assert r.returncode == 2


@pytest.mark.gpu
@pytest.mark.parametrize("kernel,split", [("spmv", "rowwise"), ("spmv", "merge"), ("spmm", "merge"),
                                          ("sddmm", "rowwise"), ("fused_spmv_axpy", "rowwise"), ("axpy", "rowwise")])
def test_cli_runs_and_checks(tmp_path, kernel, split):
    path = tmp_path / "edge.bin"
    m = M.edge_matrix()
    M.write_tgm1(str(path), m)
    r = _run("--kernel", kernel, "--matrix", str(path), "--split", split, "--tpr", "4", "--unroll", "2",
             "--vec", "2", "--block", "128", "--iters", "3", "--warmup", "1")
    assert r.returncode == 0, r.stderr
    d = json.loads(r.stdout.strip().splitlines()[-1])
    for key in ("kernel", "config", "backend", "matrix", "rows", "cols", "nnz", "ms_mean", "ms_min", "gflops",
                "bandwidth_gbs", "max_abs_err", "max_rel_err"):
        assert key in d
    assert d["rows"] == m.rows and d["nnz"] == m.nnz and d["ms_min"] > 0
    assert d["max_abs_err"] <= 1e-10, d
