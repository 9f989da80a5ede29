"""The C ABI library: loads without a GPU, exports every declared symbol, validates
schedules and sizes workspaces (no compute calls here)."""

from __future__ import annotations

import ctypes
import subprocess

import numpy as np
import pytest

from tilegen_b200 import lib


def test_library_loads_and_reports_version():
    assert "sm_100a" in lib.version()


def test_every_header_symbol_is_exported_and_typed():
    declared = set(lib.header_symbols())
    assert len(declared) == 49
    assert declared == set(lib.SIGNATURES)
    out = subprocess.run(["nm", "-D", "--defined-only", lib.lib_path()], capture_output=True, text=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    assert declared <= exported, sorted(declared - exported)
    L = lib.load()
    for name in declared:
        assert getattr(L, name) is not None


def test_reference_launcher_signatures_match_reference_abi():
    """launch_* argument lists are those of tilegen/verify.py:166-173."""
    import ctypes as C

    P, I64, F64 = C.c_void_p, C.c_int64, C.c_double
    assert lib.SIGNATURES["launch_spmv"][1] == [P, P, P, P, P, I64, I64, I64]
    assert lib.SIGNATURES["launch_spmm"][1] == [P, P, P, P, P, I64, I64, I64, I64]
    assert lib.SIGNATURES["launch_sddmm"][1] == [P, P, P, P, P, P, I64, I64, I64, I64]
    assert lib.SIGNATURES["launch_fused_spmv_axpy"][1] == [P, P, P, P, P, P, F64, F64, I64, I64, I64]
    assert lib.SIGNATURES["launch_axpy"][1] == [P, P, P, F64, F64, I64]


def test_default_schedule_is_reference_baseline():
    s = lib.default_schedule().as_dict()
    assert (s["tile"], s["threads_per_row"], s["unroll"], s["vector_width"], s["block_size"]) == (32, 1, 1, 1, 128)


@pytest.mark.parametrize("field,value,msg", [
    ("threads_per_row", 3, "threads_per_row"),
    ("unroll", 3, "unroll"),
    ("vector_width", 8, "vector_width"),
    ("block_size", 100, "block_size"),
    ("block_size", 1024, "block_size"),
    ("split", 7, "split"),
])
def test_invalid_schedules_are_rejected(field, value, msg):
    s = lib.default_schedule()
    setattr(s, field, value)
    with pytest.raises(lib.TgError) as ei:
        lib.validate_schedule(s)
    assert ei.value.status == lib.TG_EINVAL
    assert msg in str(ei.value)


def test_block_not_divisible_by_tpr_is_rejected():
    s = lib.default_schedule()
    s.threads_per_row, s.block_size = 32, 96 + 16
    with pytest.raises(lib.TgError):
        lib.validate_schedule(s)


def test_set_and_get_schedule_roundtrip():
    old = lib.get_schedule()
    s = lib.default_schedule()
    s.tile, s.threads_per_row, s.unroll = 64, 8, 2
    lib.set_schedule(s)
    got = lib.get_schedule().as_dict()
    assert (got["tile"], got["threads_per_row"], got["unroll"]) == (64, 8, 2)
    lib.set_schedule(old)


def test_workspace_sizes():
    L = lib.load()
    s = lib.default_schedule()
    assert L.tg_spmv_workspace_bytes(1000, 10000, ctypes.byref(s)) == 0  # rowwise needs none
    s.split = lib.TG_SPLIT_MERGE
    n = L.tg_spmv_workspace_bytes(1000, 10000, ctypes.byref(s))
    assert n > 0 and n % 256 == 0
    assert L.tg_spmv_workspace_bytes(1000, 0, ctypes.byref(s)) == 0
    assert L.tg_spmm_workspace_bytes(1000, 10000, 128, ctypes.byref(s)) > n
    assert L.tg_sddmm_workspace_bytes(1000, 10000, 64, ctypes.byref(s)) > 0


def test_null_arguments_fail_without_touching_the_device():
    L = lib.load()
    s = lib.default_schedule()
    assert L.tg_spmv_f64(None, None, None, ctypes.byref(s), None, 0, None) == lib.TG_EINVAL
    bad = lib.TgCsr(-1, 4, 0, 0, 0, 0)
    assert L.tg_spmv_f64(ctypes.byref(bad), None, None, ctypes.byref(s), None, 0, None) == lib.TG_EINVAL
    assert "negative size" in lib.last_error()


def test_renumber_columns_rejects_bad_bounds():
    L = lib.load()
    b = np.array([0, 10, 5], dtype=np.int64)  # decreasing
    assert L.tg_renumber_columns(None, None, 0, b.ctypes.data, 2, 32, None) == lib.TG_EINVAL
    b = np.array([0, 40], dtype=np.int64)  # shard longer than the stride allows
    assert L.tg_renumber_columns(None, None, 0, b.ctypes.data, 1, 32, None) == lib.TG_EINVAL
    b = np.array([0, 20], dtype=np.int64)
    assert L.tg_renumber_columns(None, None, 0, b.ctypes.data, 1, 32, None) == lib.TG_OK
