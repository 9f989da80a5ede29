"""GPU parity of the b200 kernels against the reference's outputs and the CPU oracle.

Shaped like the reference's CUDA suite (tests/test_cuda_gpu.py:32-104): every standard
kernel x the same seven schedules on the 257x257 edge matrix, compared with the
reference's SciPy float64 outputs under the reference tolerance
(8 * eps * max_row_nnz * max|ref| + 1e-12, tilegen/verify.py:510-514) and, per
north_star, a relative error <= 1e-9 for fp64 / <= 1e-4 for fp32 accumulation with the
relative error defined as |d| / max(|ref|, 1e-3 * max|ref|).  Then the merge split, the
reference-ABI launchers, corpus and BASELINE matrices at full size, and edge cases.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from oracle import oracle as O
from tilegen_b200 import codegen as cg
from tilegen_b200 import device as D
from tilegen_b200 import lib
from tilegen_b200 import matrices as M
from tilegen_b200.verify import inputs_for, run_kernel, run_launcher, tolerance, verify

from conftest import edge_data

pytestmark = pytest.mark.gpu

KERNELS = ["spmv", "spmm", "sddmm", "fused_spmv_axpy", "axpy"]

# tests/test_cuda_gpu.py:36-44
REF_SCHEDULES = [
    cg.Config(tile_size=32, threads_per_row=1, unroll=1, vector_width=1, block_size=128),
    cg.Config(tile_size=32, threads_per_row=2, unroll=2, vector_width=1, block_size=128),
    cg.Config(tile_size=64, threads_per_row=4, unroll=4, vector_width=2, block_size=256),
    cg.Config(tile_size=128, threads_per_row=8, unroll=2, vector_width=2, block_size=512),
    cg.Config(tile_size=32, threads_per_row=32, unroll=8, vector_width=2, block_size=512),
    cg.Config(tile_size=1, threads_per_row=4, unroll=1, vector_width=1, block_size=128),
    cg.Config(tile_size=256, threads_per_row=1, unroll=4, vector_width=1, block_size=256),
]
B200_SCHEDULES = [
    cg.Config(split="merge", block_size=256),
    cg.Config(split="merge", block_size=128, threads_per_row=8, unroll=4, vector_width=4, chunk_nnz=64),
    cg.Config(split="merge", block_size=512, threads_per_row=32, unroll=2, vector_width=2, chunk_nnz=16),
    cg.Config(tile_size=64, threads_per_row=16, unroll=4, vector_width=4, block_size=256),
    cg.Config(split="stream", unroll=1, block_size=256),
    cg.Config(split="stream", unroll=2, block_size=256),
    cg.Config(split="stream", unroll=4, block_size=128),
    cg.Config(split="stream", unroll=8, block_size=256),
]
ALL = REF_SCHEDULES + B200_SCHEDULES
IDS = ["%s-T%d-TPR%d-U%d-V%d-B%d" % (c.split, c.tile_size, c.threads_per_row, c.unroll, c.vector_width, c.block_size)
       for c in ALL]
STREAM = [c for c in B200_SCHEDULES if c.split == "stream"]


def rel_err(out, ref):
    out, ref = np.asarray(out, np.float64).ravel(), np.asarray(ref, np.float64).ravel()
    if ref.size == 0:
        return 0.0
    floor = 1e-3 * max(np.abs(ref).max(), 1e-300)
    return float((np.abs(out - ref) / np.maximum(np.abs(ref), floor)).max())


def check_f64(out, ref, A):
    out, ref = np.asarray(out).ravel(), np.asarray(ref).ravel()
    tol = tolerance(A, ref)
    d = float(np.abs(out - ref).max()) if ref.size else 0.0
    assert d <= tol, "max abs err %.3g > tol %.3g" % (d, tol)
    assert rel_err(out, ref) <= 1e-9


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    lib.load()
    yield


@pytest.mark.parametrize("kernel", KERNELS)
@pytest.mark.parametrize("cfg", ALL, ids=IDS)
def test_kernel_matches_float64_reference(kernel, cfg, edge, edge_csr):
    out = run_kernel(cg.generate(kernel, cfg), edge_csr, edge_data(edge), K=8)
    check_f64(out, edge["ref_" + kernel], edge_csr)


@pytest.mark.parametrize("kernel", KERNELS)
@pytest.mark.parametrize("cfg", [REF_SCHEDULES[0], REF_SCHEDULES[3], B200_SCHEDULES[0], B200_SCHEDULES[1],
                                 B200_SCHEDULES[5]],
                         ids=["T32", "T128-TPR8", "merge256", "merge128", "stream"])
def test_fp32_accumulation_within_1e_4(kernel, cfg, edge, edge_csr):
    c = cg.Config(**{**cfg.to_dict(), "dtype": "f32"})
    out = run_kernel(cg.generate(kernel, c), edge_csr, edge_data(edge), K=8)
    assert rel_err(out, edge["ref_" + kernel]) <= 1e-4
    # and against the reference's own fp32 OpenMP backend
    assert rel_err(out, edge["omp_%s_f32" % kernel]) <= 1e-4


@pytest.mark.parametrize("kernel", KERNELS)
@pytest.mark.parametrize("split", ["rowwise", "merge", "stream"])
def test_injected_bug_is_caught(kernel, split, edge_csr):
    cfg = cg.Config(tile_size=32, threads_per_row=4, unroll=2, vector_width=1, block_size=256, inject_bug=True,
                    split=split)
    res = verify(kernel, cfg, edge_csr, K=8)
    assert not res.ok and res.max_abs_err > res.tolerance, res
    good = verify(kernel, cg.Config(**{**cfg.to_dict(), "inject_bug": False}), edge_csr, K=8)
    assert good.ok, good


@pytest.mark.parametrize("kernel", KERNELS)
@pytest.mark.parametrize("cfg", [REF_SCHEDULES[0], REF_SCHEDULES[4], B200_SCHEDULES[0]], ids=["T32", "TPR32", "merge"])
def test_reference_abi_launchers(kernel, cfg, edge, edge_csr):
    """launch_<name> with device pointers and the process-global schedule, exactly as
    the reference's verify.run_kernel calls a generated CUDA object."""
    sched = cg.generate(kernel, cfg).sched
    out = run_launcher(kernel, edge_csr, edge_data(edge), K=8, sched=sched)
    check_f64(out, edge["ref_" + kernel], edge_csr)
    lib.set_schedule(lib.default_schedule())


@pytest.mark.parametrize("split", ["rowwise", "merge", "stream"])
def test_corner_cases(corner, split):
    for name in ("bug4", "empty_row3", "zeros2", "small3"):
        shape = tuple(int(s) for s in corner[name + "_shape"])
        A = M.CSR(corner[name + "_indptr"], corner[name + "_indices"], corner[name + "_data"], shape, name)
        data = tuple(corner[name + "_" + k] for k in ("x", "w", "B", "U", "V")) + (0.7, -1.3)
        for kernel in KERNELS:
            out = run_kernel(cg.generate(kernel, cg.Config(unroll=2, split=split)), A, data, K=8)
            check_f64(out, corner[name + "_ref_" + kernel], A)
        if name == "zeros2":
            out = run_kernel(cg.generate("spmv", cg.Config(unroll=4, split=split)), A, data, K=8)
            assert np.all(out == 0.0)  # exact zero (tests/test_verify.py:39-43)


@pytest.mark.parametrize("split", ["rowwise", "merge", "stream"])
def test_empty_and_degenerate_shapes(split):
    dev = torch.device("cuda")
    s = cg.generate("spmv", cg.Config(split=split)).sched
    # nnz == 0: every row is zero; rows == 0: nothing to do
    for rows, cols in ((5, 7), (0, 3), (1, 1)):
        A = D.DeviceCSR(torch.zeros(rows + 1, dtype=torch.int64, device=dev), torch.zeros(0, dtype=torch.int64, device=dev),
                        torch.zeros(0, dtype=torch.float64, device=dev), (rows, cols))
        y = torch.full((rows,), 7.0, dtype=torch.float64, device=dev)
        D.spmv(A, torch.ones(cols, dtype=torch.float64, device=dev), y, sched=s)
        assert torch.all(y == 0)
        C = torch.full((rows, 4), 3.0, dtype=torch.float64, device=dev)
        D.spmm(A, torch.ones((cols, 4), dtype=torch.float64, device=dev), C, sched=s)
        assert torch.all(C == 0)
    # trailing and leading empty rows around a single nonzero
    m = M.CSR(np.array([0, 0, 0, 1, 1, 1], np.int64), np.array([2], np.int64), np.array([5.0]), (5, 3))
    x = np.array([1.0, 2.0, 3.0])
    out = run_kernel(cg.generate("spmv", cg.Config(split=split)), m, (x, x, None, None, None, 1.0, 1.0))
    assert np.array_equal(out, [0, 0, 15.0, 0, 0])


@pytest.mark.parametrize("cls", M.corpus_classes())
@pytest.mark.parametrize("cfg", [cg.Config(threads_per_row=8, unroll=2, vector_width=2, block_size=256),
                                 cg.Config(split="merge", block_size=256),
                                 cg.Config(split="stream", unroll=2)], ids=["TPR8", "merge", "stream"])
def test_corpus_classes_spmv_full(cls, cfg):
    m = M.make_matrix(cls)
    x = inputs_for("spmv", m, 8, 7)[0]
    out = run_kernel(cg.generate("spmv", cfg), m, (x, None, None, None, None, 1.0, 1.0))
    check_f64(out, O.spmv(m, x), m)


@pytest.mark.parametrize("name", ["c1", "c2", "c3"])
@pytest.mark.parametrize("cfg", [cg.Config(tile_size=64, threads_per_row=16, unroll=2, vector_width=2, block_size=256),
                                 cg.Config(split="merge", block_size=256),
                                 cg.Config(split="stream", unroll=1),
                                 cg.Config(split="stream", unroll=8)], ids=["TPR16", "merge", "stream1", "stream8"])
def test_baseline_spmv_configs_full_size(name, cfg):
    m = M.baseline_matrix(name)
    x = np.random.default_rng(11).uniform(-1, 1, m.cols)
    out = run_kernel(cg.generate("spmv", cfg), m, (x, None, None, None, None, 1.0, 1.0))
    check_f64(out, O.spmv(m, x), m)


def _long_row_matrix():
    """Rows of 1..3 nonzeros around three long rows (60000, 7001 and 2049 nonzeros), so
    rows span many merge chunks, start/end mid-chunk, and chunk boundaries fall on row
    boundaries too."""
    rng = np.random.default_rng(17)
    n = 70000
    lens = rng.integers(0, 4, n)
    lens[5], lens[40000], lens[n - 1] = 60000, 7001, 2049
    indptr = np.zeros(n + 1, np.int64)
    np.cumsum(lens, out=indptr[1:])
    idx = np.concatenate([np.sort(rng.choice(n, size=L, replace=False)) if L else np.zeros(0, np.int64)
                          for L in lens]).astype(np.int64)
    return M.CSR(indptr, idx, rng.uniform(-1, 1, idx.size), (n, n), "longrows")


@pytest.mark.parametrize("cfg", [cg.Config(split="merge", block_size=128), cg.Config(split="merge", block_size=256),
                                 cg.Config(split="merge", threads_per_row=32, unroll=4, vector_width=2, chunk_nnz=32),
                                 cg.Config(threads_per_row=32, unroll=4, vector_width=2),
                                 cg.Config(split="stream", unroll=1), cg.Config(split="stream", unroll=8)],
                         ids=["merge128", "merge256", "merge-c32", "rowwise", "stream1", "stream8"])
def test_long_rows_spanning_chunks(cfg):
    m = _long_row_matrix()
    data = inputs_for("spmm", m, 16, 3)
    x, w, B, U, V, a, b = data
    for kernel, ref in (("spmv", O.spmv(m, x)), ("fused_spmv_axpy", O.fused_spmv_axpy(m, x, w, a, b)),
                        ("spmm", O.spmm(m, B)), ("sddmm", O.sddmm(m, U, V))):
        out = run_kernel(cg.generate(kernel, cfg), m, data, K=16)
        check_f64(out, ref, m)


def test_merge_results_are_deterministic():
    m = _long_row_matrix()
    data = inputs_for("spmm", m, 16, 3)
    g = cg.generate("spmv", cg.Config(split="merge"))
    a = run_kernel(g, m, data)
    b = run_kernel(g, m, data)
    assert np.array_equal(a, b)
    g = cg.generate("spmm", cg.Config(split="merge", chunk_nnz=32))
    assert np.array_equal(run_kernel(g, m, data, K=16), run_kernel(g, m, data, K=16))
    g = cg.generate("spmv", cg.Config(split="stream", unroll=2))
    assert np.array_equal(run_kernel(g, m, data), run_kernel(g, m, data))


@pytest.mark.parametrize("cfg", [cg.Config(split="stream", unroll=4), cg.Config(split="merge", block_size=128),
                                 cg.Config(split="merge", block_size=256)], ids=["stream", "merge128", "merge256"])
def test_plan_reuse_flag(cfg):
    """TG_FLAG_REUSE_PLAN skips the analysis pass on a workspace planned for the same
    matrix; results are identical to a planned call (the merge split's arrival counters
    are back at zero after every call)."""
    m = _long_row_matrix()
    A = D.DeviceCSR.from_host(m, "cuda")
    x = torch.as_tensor(np.random.default_rng(3).uniform(-1, 1, m.cols)).cuda()
    s = cg.generate("spmv", cfg).sched
    L = lib.load()
    nb = L.tg_spmv_workspace_bytes(m.rows, m.nnz, ctypes.byref(s))
    ws = torch.zeros(nb, dtype=torch.uint8, device="cuda")
    y1 = D.spmv(A, x, sched=s, workspace=ws)
    s.flags |= lib.TG_FLAG_REUSE_PLAN
    y2 = D.spmv(A, x, sched=s, workspace=ws)
    y3 = D.spmv(A, x, sched=s, workspace=ws)
    assert torch.equal(y1, y2) and torch.equal(y2, y3)
    check_f64(y1.cpu().numpy(), O.spmv(m, x.cpu().numpy()), m)


@pytest.mark.parametrize("K", [1, 3, 8, 64, 100, 128, 600])
@pytest.mark.parametrize("split", ["rowwise", "merge"])
def test_dense_widths(K, split):
    m = M.baseline_matrix("c3", scale=0.02)
    data = inputs_for("spmm", m, K, 5)
    for dtype in ("f64", "f32"):
        cfg = cg.Config(threads_per_row=32, unroll=2, vector_width=4, split=split, dtype=dtype)
        for kernel, ref in (("spmm", O.spmm(m, data[2])), ("sddmm", O.sddmm(m, data[3], data[4]))):
            out = run_kernel(cg.generate(kernel, cfg), m, data, K=K)
            if dtype == "f64":
                check_f64(out, ref, m)
            else:
                assert rel_err(out, ref) <= 1e-4, (kernel, K, split)


def _wide_matrix():
    """2000 rows over 1,000,000 columns (power-law row lengths, a few long rows): a dense
    operand of 1M rows, larger than L2 for every K here."""
    rng = np.random.default_rng(31)
    rows, cols = 2000, 1_000_000
    lens = np.minimum(np.floor(1.0 / rng.uniform(size=rows)).astype(np.int64), 3000)
    lens[7] = 2600
    indptr = np.zeros(rows + 1, np.int64)
    np.cumsum(lens, out=indptr[1:])
    idx = np.concatenate([np.sort(rng.choice(cols, size=L, replace=False)) for L in lens]).astype(np.int64)
    return M.CSR(indptr, idx, rng.uniform(-1, 1, idx.size), (rows, cols), "wide")


@pytest.mark.parametrize("K", [8, 24, 40, 64, 100])
@pytest.mark.parametrize("split", ["rowwise", "merge"])
def test_wide_dense_operand(K, split):
    """SpMM and SDDMM gathering from a 1M-row dense operand (SpMM with K above one lane
    group's width runs one launch per column slab) against the oracle, fp64 and fp32."""
    m = _wide_matrix()
    data = inputs_for("spmm", m, K, 6)
    for dtype in ("f64", "f32"):
        cfg = cg.Config(threads_per_row=32, unroll=2, vector_width=4, split=split, dtype=dtype)
        for kernel, ref in (("spmm", O.spmm(m, data[2])), ("sddmm", O.sddmm(m, data[3], data[4]))):
            out = run_kernel(cg.generate(kernel, cfg), m, data, K=K)
            if dtype == "f64":
                check_f64(out, ref, m)
            else:
                assert rel_err(out, ref) <= 1e-4, (kernel, K, split)


def _mixed_group_matrix():
    """Row groups of 8 that share a column list (8x8 blocks) next to groups that do not
    (one row of a group differs in one column, or in its length), a partial last group
    and empty rows."""
    rng = np.random.default_rng(41)
    rows = []
    for g in range(40):
        cols = np.sort(rng.choice(5000, size=int(rng.integers(0, 40)), replace=False))
        grp = [cols.copy() for _ in range(8)]
        if g % 3 == 1 and cols.size:
            grp[5] = np.sort(np.unique(np.append(cols[:-1], (cols[-1] + 1) % 5000)))
        elif g % 3 == 2:
            grp[2] = np.sort(rng.choice(5000, size=int(rng.integers(1, 60)), replace=False))
        rows.extend(grp)
    rows.extend([np.sort(rng.choice(5000, size=7, replace=False)) for _ in range(5)])
    indptr = np.zeros(len(rows) + 1, np.int64)
    np.cumsum([r.size for r in rows], out=indptr[1:])
    idx = np.concatenate(rows).astype(np.int64)
    return M.CSR(indptr, idx, rng.uniform(-1, 1, idx.size), (len(rows), 5000), "mixed_groups")


@pytest.mark.parametrize("K", [8, 100, 128, 300])
@pytest.mark.parametrize("name", ["blocked", "mixed", "edge", "c3"])
def test_block_split_spmm(K, name, edge_csr):
    """SpMM over row groups (TG_SPLIT_BLOCK): groups of 8 rows with one column list share
    each gathered B row; the rest go row by row.  Against the oracle in fp64 and fp32;
    the plan (group flags) reused on a second call gives identical output."""
    m = {"blocked": lambda: M.make_matrix("blocked"), "mixed": _mixed_group_matrix, "edge": lambda: edge_csr,
         "c3": lambda: M.baseline_matrix("c3", scale=0.02)}[name]()
    data = inputs_for("spmm", m, K, 9)
    ref = O.spmm(m, data[2])
    for dtype in ("f64", "f32"):
        cfg = cg.Config(split="block", dtype=dtype)
        out = run_kernel(cg.generate("spmm", cfg), m, data, K=K)
        if dtype == "f64":
            check_f64(out, ref, m)
        else:
            assert rel_err(out, ref) <= 1e-4, (name, K)
    # plan reuse
    dev = torch.device("cuda")
    A = D.DeviceCSR.from_host(m, dev)
    Bd = torch.as_tensor(data[2]).to(dev)
    s = cg.generate("spmm", cg.Config(split="block")).sched
    L = lib.load()
    ws = torch.zeros(max(1, int(L.tg_spmm_workspace_bytes(m.rows, m.nnz, K, ctypes.byref(s)))), dtype=torch.uint8,
                     device=dev)
    C1 = D.spmm(A, Bd, sched=s, workspace=ws)
    s.flags |= lib.TG_FLAG_REUSE_PLAN
    C2 = D.spmm(A, Bd, sched=s, workspace=ws)
    assert torch.equal(C1, C2)


def test_block_split_matches_rowwise_bitwise():
    """Each row is summed over its nonzeros in index order on both paths, so the block
    split's output equals the rowwise kernel's bit for bit."""
    m = M.make_matrix("blocked")
    data = inputs_for("spmm", m, 128, 2)
    for dtype in ("f64", "f32"):
        a = run_kernel(cg.generate("spmm", cg.Config(split="block", dtype=dtype)), m, data, K=128)
        b = run_kernel(cg.generate("spmm", cg.Config(threads_per_row=32, vector_width=4, dtype=dtype)), m, data,
                       K=128)
        assert np.array_equal(a, b), dtype


def test_misaligned_operands_use_safe_paths():
    """Views that start one element into their allocation break 16-byte alignment; the
    library must switch to scalar loads (no TMA, V=1) and stay correct."""
    m = M.baseline_matrix("c1", scale=0.01)
    dev = torch.device("cuda")
    ip = torch.as_tensor(m.indptr).to(dev)
    ix = torch.cat([torch.zeros(1, dtype=torch.int64), torch.as_tensor(m.indices)]).to(dev)[1:]
    dv = torch.cat([torch.zeros(1, dtype=torch.float64), torch.as_tensor(m.data)]).to(dev)[1:]
    assert ix.data_ptr() % 16 == 8
    A = D.DeviceCSR(ip, ix, dv, m.shape)
    x = np.random.default_rng(2).uniform(-1, 1, m.cols)
    ref = O.spmv(m, x)
    for cfg in (cg.Config(threads_per_row=8, vector_width=4, unroll=2), cg.Config(split="merge")):
        y = D.spmv(A, torch.as_tensor(x).to(dev), sched=cg.generate("spmv", cfg))
        check_f64(y.cpu().numpy(), ref, m)


def test_bounds_check_reports_bad_index_without_computing():
    dev = torch.device("cuda")
    ip = torch.tensor([0, 2, 3], dtype=torch.int64, device=dev)
    ix = torch.tensor([0, 5, 1], dtype=torch.int64, device=dev)  # 5 >= cols
    A = D.DeviceCSR(ip, ix, torch.ones(3, dtype=torch.float64, device=dev), (2, 3))
    y = torch.full((2,), -1.0, dtype=torch.float64, device=dev)
    with pytest.raises(lib.TgError) as ei:
        D.spmv(A, torch.ones(3, dtype=torch.float64, device=dev), y,
               sched=cg.generate("spmv", cg.Config(bounds_check=True)))
    assert ei.value.status == lib.TG_EBOUNDS and "out of range" in str(ei.value)
    assert torch.all(y == -1.0)
    ix[1] = 2
    D.spmv(A, torch.ones(3, dtype=torch.float64, device=dev), y, sched=cg.generate("spmv", cg.Config(bounds_check=True)))
    assert torch.allclose(y, torch.tensor([2.0, 1.0], dtype=torch.float64, device=dev))


def test_workspace_too_small_is_an_error():
    m = M.baseline_matrix("c1", scale=0.01)
    A = D.DeviceCSR.from_host(m, "cuda")
    s = cg.generate("spmv", cg.Config(split="merge")).sched
    L = lib.load()
    x = torch.zeros(m.cols, dtype=torch.float64, device="cuda")
    y = torch.zeros(m.rows, dtype=torch.float64, device="cuda")
    st = L.tg_spmv_f64(ctypes.byref(A.desc()), x.data_ptr(), y.data_ptr(), ctypes.byref(s), None, 0, None)
    assert st == lib.TG_ENOMEM and "workspace" in lib.last_error()


@pytest.mark.parametrize("split,scale", [("rowwise", 0.05), ("merge", 0.05), ("merge", 0.3)])
def test_c5_spmm_sddmm_scaled(split, scale):
    """C5's generator at 5 % and 30 % of its rows (300k rows, ~4.8M nonzeros at 0.3), every
    output element against the oracle (fp32 bar)."""
    m = M.baseline_matrix("c5", scale=scale).astype(np.float32)
    rng = np.random.default_rng(8)
    B = rng.uniform(-1, 1, (m.cols, 128)).astype(np.float32)
    U = rng.uniform(-1, 1, (m.rows, 64)).astype(np.float32)
    V = rng.uniform(-1, 1, (m.cols, 64)).astype(np.float32)
    cfg = cg.Config(threads_per_row=32, unroll=4, vector_width=4, split=split, dtype="f32")
    A = D.DeviceCSR.from_host(m, "cuda", torch.float32)
    C = D.spmm(A, torch.as_tensor(B).cuda(), sched=cg.generate("spmm", cfg)).cpu().numpy()
    assert rel_err(C, O.spmm(m.astype(np.float64), B.astype(np.float64))) <= 1e-4
    out = D.sddmm(A, torch.as_tensor(U).cuda(), torch.as_tensor(V).cuda(), sched=cg.generate("sddmm", cfg)).cpu().numpy()
    assert rel_err(out, O.sddmm(m.astype(np.float64), U.astype(np.float64), V.astype(np.float64))) <= 1e-4
