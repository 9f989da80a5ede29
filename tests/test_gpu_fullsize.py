"""Parity at the BASELINE sizes through size-independent properties (the oracle finishes
in seconds only on smaller cases): the C4 power iteration against the oracle's OpenMP
SpMV loop at full size, SpMV linearity at full size, and C5 SpMM / SDDMM through
checksums (C·1 = A·(B·1); Σ out = Σ_i U_i·(A V)_i) plus sampled exact rows / nonzeros."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import oracle as O
from tilegen_b200 import codegen as cg
from tilegen_b200 import device as D
from tilegen_b200 import lib
from tilegen_b200 import matrices as M
from tilegen_b200.power import PowerIteration, uniform_bounds

pytestmark = pytest.mark.gpu


def rel(out, ref):
    out, ref = np.asarray(out, np.float64).ravel(), np.asarray(ref, np.float64).ravel()
    floor = 1e-3 * max(np.abs(ref).max(), 1e-300)
    return float((np.abs(out - ref) / np.maximum(np.abs(ref), floor)).max())


@pytest.fixture(scope="module")
def c4():
    return M.baseline_matrix("c4")


def test_c4_full_power_iteration_matches_oracle(c4):
    """20 power iterations on the 8M-row, 256M-nonzero C4 matrix (the bench workload)
    against the same recurrence on the host with the oracle's OpenMP SpMV; fp64 bar."""
    n = c4.rows
    x0 = np.random.default_rng([7, 0]).uniform(-1.0, 1.0, size=n)
    dev = torch.device("cuda")
    s = lib.default_schedule()
    s.threads_per_row, s.unroll, s.vector_width, s.block_size = 4, 2, 2, 256
    pi = PowerIteration(torch.as_tensor(c4.indptr).to(dev), torch.as_tensor(c4.indices).to(dev),
                        torch.as_tensor(c4.data).to(dev), uniform_bounds(n, 1), 0, sched=s)
    pi.set_x0(torch.as_tensor(x0).to(dev))
    pi.iterate(20)
    x, lam = pi.result()
    xh = x0 / np.sqrt(np.dot(x0, x0))
    y = np.empty(n)
    nrm = 0.0
    for _ in range(20):
        O.spmv_omp(c4, xh, out=y)
        nrm = float(np.sqrt(np.dot(y, y)))
        xh = y / nrm
    assert rel(x.cpu().numpy(), xh) <= 1e-9
    assert abs(float(lam) - nrm) <= 1e-9 * nrm


@pytest.mark.parametrize("split", ["rowwise", "merge"])
def test_c4_full_spmv_is_linear(c4, split):
    """A(a x1 + b x2) = a A x1 + b A x2 on the full C4 matrix, on the device."""
    dev = torch.device("cuda")
    A = D.DeviceCSR.from_host(c4, dev)
    g = torch.Generator(device=dev)
    g.manual_seed(3)
    x1 = torch.rand(c4.cols, dtype=torch.float64, device=dev, generator=g) * 2 - 1
    x2 = torch.rand(c4.cols, dtype=torch.float64, device=dev, generator=g) * 2 - 1
    a, b = 0.75, -1.5
    sch = cg.generate("spmv", cg.Config(threads_per_row=4, unroll=2, vector_width=2, block_size=256, split=split))
    y1 = D.spmv(A, x1, sched=sch)
    y2 = D.spmv(A, x2, sched=sch)
    y3 = D.spmv(A, a * x1 + b * x2, sched=sch)
    assert rel((a * y1 + b * y2).cpu().numpy(), y3.cpu().numpy()) <= 1e-12


@pytest.fixture(scope="module")
def c5():
    return M.baseline_matrix("c5")


def test_c5_full_spmm_checksum_and_sampled_rows(c5):
    dev = torch.device("cuda")
    rng = np.random.default_rng(21)
    B = rng.uniform(-1.0, 1.0, size=(c5.cols, 128)).astype(np.float32)
    A32 = D.DeviceCSR.from_host(c5, dev, torch.float32)
    sch = cg.generate("spmm", cg.Config(split="merge", threads_per_row=32, unroll=4, vector_width=4, block_size=128,
                                        dtype="f32"))
    C = D.spmm(A32, torch.as_tensor(B).to(dev), sched=sch)
    # checksum of checksums: C 1 = A (B 1), in fp64 on the host with the fp32-rounded values
    a64 = c5.astype(np.float32).astype(np.float64)
    want = O.spmv_omp(a64, B.astype(np.float64).sum(axis=1))[0]
    got = C.double().sum(dim=1).cpu().numpy()
    assert rel(got, want) <= 1e-4
    rows = rng.choice(c5.rows, size=2000, replace=False)
    Cs = C[torch.as_tensor(rows, device=dev)].double().cpu().numpy()
    for k, r in enumerate(rows):
        p0, p1 = a64.indptr[r], a64.indptr[r + 1]
        ref = a64.data[p0:p1] @ B[a64.indices[p0:p1]].astype(np.float64) if p1 > p0 else np.zeros(128)
        assert rel(Cs[k], ref) <= 1e-4


def test_c5_full_sddmm_checksum_and_sampled_nonzeros(c5):
    dev = torch.device("cuda")
    rng = np.random.default_rng(22)
    U = rng.uniform(-1.0, 1.0, size=(c5.rows, 64)).astype(np.float32)
    V = rng.uniform(-1.0, 1.0, size=(c5.cols, 64)).astype(np.float32)
    A32 = D.DeviceCSR.from_host(c5, dev, torch.float32)
    sch = cg.generate("sddmm", cg.Config(split="merge", threads_per_row=8, unroll=1, vector_width=4, block_size=128,
                                         dtype="f32"))
    out = D.sddmm(A32, torch.as_tensor(U).to(dev), torch.as_tensor(V).to(dev), sched=sch).double().cpu().numpy()
    a64 = c5.astype(np.float32).astype(np.float64)
    S = a64.to_scipy()
    want = float(np.einsum("ik,ik->", U.astype(np.float64), S @ V.astype(np.float64)))
    assert abs(out.sum() - want) <= 1e-4 * np.abs(out).sum()
    rows = np.repeat(np.arange(a64.rows), np.diff(a64.indptr))
    pick = rng.choice(a64.nnz, size=20000, replace=False)
    ref = a64.data[pick] * np.einsum("ik,ik->i", U[rows[pick]].astype(np.float64),
                                     V[a64.indices[pick]].astype(np.float64))
    assert rel(out[pick], ref) <= 1e-4
