"""Autotuner (mirror of the reference's tests/test_autotune.py: pruning with reasons, tune
smoke, output schema) plus the b200 additions (split dimension, compulsory bytes)."""

from __future__ import annotations

import json
import os
import random

import numpy as np
import pytest

from tilegen_b200 import autotune as at
from tilegen_b200.codegen import Config
from tilegen_b200.matrices import CSR


def _small_matrix():
    # the reference test's 4x4 matrix (tests/test_autotune.py:22-27)
    return {"indptr": np.array([0, 2, 3, 4, 6], dtype=np.int64),
            "indices": np.array([0, 1, 2, 2, 1, 3], dtype=np.int64),
            "data": np.array([1.0, 2.0, 3.0, 4.0, 5.0, 6.0]), "shape": (4, 4), "class_name": "tiny"}


def test_space_and_prune_counts_match_reference():
    assert len(at.enumerate_configs()) == 720
    assert len(at.legal_configs()) == 540
    assert len(at.prune_log()) == 180
    pruned = [(c, r) for c, r in at.enumerate_configs() if r is not None]
    assert all(isinstance(r, str) and r for _, r in pruned)


def test_illegal_rules():
    assert at.illegal_reason(Config(threads_per_row=8, block_size=4)) is not None
    assert at.illegal_reason(Config(vector_width=4, unroll=2)) is not None
    assert at.illegal_reason(Config(threads_per_row=32, block_size=128)) is None
    assert at.illegal_reason(Config(threads_per_row=16, block_size=128)) is None  # b200 instance
    assert "no b200 instance" in at.illegal_reason(Config(threads_per_row=64, block_size=128))
    assert "unknown" in at.illegal_reason(Config(split="diagonal"))
    assert all(at.illegal_reason(c) is None for c in at.legal_configs(at.B200_SEARCH_SPACE, at.SPLITS))


def test_split_dimension():
    legal = at.legal_configs(at.B200_SEARCH_SPACE, at.SPLITS)
    assert {c.split for c in legal} == set(at.SPLITS)
    assert len(legal) == len(at.SPLITS) * len(at.legal_configs(at.B200_SEARCH_SPACE))
    # distinct hashes: a rowwise config keeps the reference's key, the others differ
    hashes = {c.hash() for c in legal}
    assert len(hashes) == len(legal)


@pytest.mark.parametrize("mode", ["random", "coordinate"])
def test_candidates_start_at_baseline(mode):
    c = at._candidate_configs(12, mode, random.Random(0), "spmv", at.SPLITS)
    assert c[0].hash() == at.BASELINE.hash()
    assert len(c) == 12 and len({x.hash() for x in c}) == 12
    assert all(at.illegal_reason(x) is None for x in c)
    # no stream variants for SpMM (its stream split is the merge kernel), no block variants
    # outside SpMM (the block split is an SpMM mapping)
    d = at._candidate_configs(200, "random", random.Random(1), "spmm", at.SPLITS, dtype="f32")
    assert all(x.split != "stream" and x.dtype == "f32" for x in d)
    assert any(x.split == "block" for x in d)
    assert all(x.split != "block" for x in at._candidate_configs(200, "random", random.Random(1), "spmv", at.SPLITS))


def test_coordinate_adds_split_variants():
    c = at._candidate_configs(100, "coordinate", random.Random(0), "spmv", at.SPLITS)
    assert {"merge", "stream"} <= {x.split for x in c}


def test_flops_bytes_compulsory():
    A = CSR(np.array([0, 2, 3, 4, 6]), np.array([0, 1, 2, 2, 1, 3]), np.ones(6), (4, 4), "tiny")
    f, ref_b, comp = at.flops_bytes("spmv", A, 8)
    assert f == 12.0
    assert comp == 8 * 5 + 16 * 6 + 8 * 4 + 8 * 4  # indptr + indices/values + x + y
    assert ref_b == 6 * 16.0 + 5 * 8.0 + 6 * 8.0 + 4 * 8.0  # tilegen/autotune.py:96-98
    _, _, c32 = at.flops_bytes("spmm", A, 128, "f32")
    assert c32 == 8 * 5 + 12 * 6 + 4 * 128 * 8


def _fake_result(cls, kernel, ms):
    rec = {"kernel": kernel, "matrix_class": cls, "rows": 4, "nnz": 6, "config": Config().to_dict(), "skipped": None,
           "ms_mean": ms, "ms_min": ms, "ms_median": ms, "gflops": 1.0, "bandwidth_gbs": 2.0, "effective_gbs": 3.0,
           "max_abs_err": 0.0, "max_rel_err": 0.0, "tolerance": 1e-12, "ok": True, "speedup_vs_naive": 1.0}
    return {"kernel": kernel, "matrix_class": cls, "baseline": at.BASELINE.to_dict(), "baseline_ms_min": ms,
            "winner": rec["config"], "winner_metrics": rec, "records": [rec]}


def test_write_outputs_schema(tmp_path):
    full = tmp_path / "full"
    at.write_outputs([_fake_result("tiny", "spmv", 0.5)], str(tmp_path), {"backend": "b200"}, at.prune_log(),
                     full_outdir=str(full))
    for name in ["autotune.json", "autotune.csv", "best_configs.json"]:
        assert os.path.exists(str(tmp_path / name))
    data = json.load(open(str(tmp_path / "autotune.json")))
    assert "results" in data and "pruned" in data and "hardware" in data and "best" in data and "top5" in data
    assert all("records" not in r for r in data["results"])
    assert data["best"]["tiny"]["spmv"]["metrics"]["effective_gbs"] == 3.0
    assert len(data["top5"]["tiny"]) <= 5
    raw = json.load(open(str(full / "autotune.json")))
    assert raw["results"][0]["records"]
    header = open(str(tmp_path / "autotune.csv")).readline().strip().split(",")
    assert header[:3] == ["matrix_class", "kernel", "split"]


@pytest.mark.gpu
def test_tune_smoke_gpu(tmp_path):
    res = at.tune("spmv", _small_matrix(), budget=4, mode="coordinate", warmup=1, iters=3,
                  splits=at.SPLITS, workdir=str(tmp_path))
    assert res["winner"] is not None
    measured = [r for r in res["records"] if r.get("ms_min")]
    assert measured and all(r["ok"] for r in measured)
    for key in ["ms_mean", "ms_min", "ms_median", "gflops", "bandwidth_gbs", "effective_gbs", "max_abs_err", "ok",
                "speedup_vs_naive"]:
        assert key in res["winner_metrics"]
    assert res["baseline"] == at.BASELINE.to_dict()
    assert res["baseline_ms_min"] is not None


@pytest.mark.gpu
@pytest.mark.parametrize("kernel", ["spmm", "sddmm", "fused_spmv_axpy"])
def test_tune_dense_kernels_gpu(kernel, edge_csr):
    res = at.tune(kernel, edge_csr, budget=5, warmup=1, iters=2, seed=3, splits=("rowwise", "merge"),
                  space=at.B200_SEARCH_SPACE, flush_l2=False)
    measured = [r for r in res["records"] if r.get("ms_min")]
    assert measured and all(r["ok"] for r in measured), [r.get("max_abs_err") for r in measured]
