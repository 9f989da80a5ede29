"""GPU parity of the power iteration (tg_power_step_f64 & co.) against the oracle."""

from __future__ import annotations

import ctypes
import time

import numpy as np
import pytest
import torch

from oracle import oracle as O
from tilegen_b200 import lib
from tilegen_b200 import matrices as M
from tilegen_b200.power import PowerIteration, nnz_balanced_bounds, uniform_bounds

pytestmark = pytest.mark.gpu


def _sched(tpr=8, u=2, v=2, b=256, split="rowwise"):
    s = lib.default_schedule()
    s.threads_per_row, s.unroll, s.vector_width, s.block_size = tpr, u, v, b
    s.split = lib.TG_SPLIT_STREAM if split == "stream" else lib.TG_SPLIT_ROWWISE
    return s


def rel(a, b):
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-300))


@pytest.mark.parametrize("tpr,u,v,split", [(4, 1, 1, "rowwise"), (4, 1, 4, "rowwise"), (8, 2, 2, "rowwise"),
                                           (16, 4, 2, "rowwise"),
                                           (32, 2, 4, "rowwise"), (4, 1, 1, "stream"), (4, 2, 2, "stream"),
                                           (4, 4, 2, "stream"), (4, 8, 2, "stream")])
def test_power_iteration_single_gpu_matches_oracle(tpr, u, v, split):
    n = 200_000
    A = M.c4_rows(0, n, n=n, per_row=32, seed=4)
    x0 = np.random.default_rng(1).uniform(-1, 1, n)
    dev = torch.device("cuda")
    pi = PowerIteration(torch.as_tensor(A.indptr).to(dev), torch.as_tensor(A.indices).to(dev),
                        torch.as_tensor(A.data).to(dev), uniform_bounds(n, 1), 0, sched=_sched(tpr, u, v, 256, split))
    pi.set_x0(torch.as_tensor(x0).to(dev))
    pi.iterate(20)
    x, lam = pi.result()
    xr, nr = O.power_iteration(A, x0, 20)
    assert rel(x.cpu().numpy(), xr) <= 1e-9
    assert abs(float(lam) - nr) <= 1e-9 * nr


@pytest.mark.parametrize("parts", [2, 3, 4, 8])
@pytest.mark.parametrize("split", ["rowwise", "stream"])
def test_sharded_layout_emulated_on_one_gpu(parts, split):
    """P shards on one device with the shard exchange done by device copies: checks the
    nnz-balanced bounds, column renumbering, padded layout and slot reduction."""
    A = M.baseline_matrix("c3", scale=0.3)  # power-law rows: unequal shards
    n = A.rows
    bounds = nnz_balanced_bounds(A.row_lengths(), parts)
    dev = torch.device("cuda")
    pis = []
    for r in range(parts):
        a, b = int(bounds[r]), int(bounds[r + 1])
        ip = A.indptr[a:b + 1] - A.indptr[a]
        sl = slice(int(A.indptr[a]), int(A.indptr[b]))
        pis.append(PowerIteration(torch.as_tensor(ip).to(dev), torch.as_tensor(A.indices[sl]).to(dev),
                                  torch.as_tensor(A.data[sl]).to(dev), bounds, r, sched=_sched(split=split),
                                  exchange=lambda x: None))
    stride = pis[0].stride

    def exchange(buf_index):
        for r in range(parts):
            src = pis[r].x[buf_index][r * stride:(r + 1) * stride]
            for q in range(parts):
                if q != r:
                    pis[q].x[buf_index][r * stride:(r + 1) * stride].copy_(src)

    x0 = np.random.default_rng(2).uniform(-1, 1, n)
    for r, pi in enumerate(pis):
        pi.set_x0(torch.as_tensor(x0[bounds[r]:bounds[r + 1]]).to(dev))
    exchange(0)
    cur = 0
    for _ in range(12):
        for pi in pis:
            pi._step(pi.x[cur], pi.shard(pi.x[1 - cur]))
        exchange(1 - cur)
        cur = 1 - cur
        for pi in pis:
            pi.cur = cur
    x = np.concatenate([pi.result()[0].cpu().numpy() for pi in pis])
    xr, nr = O.power_iteration(A, x0, 12)
    assert rel(x, xr) <= 1e-9
    lams = [float(pi.result()[1]) for pi in pis]
    assert max(abs(l - nr) for l in lams) <= 1e-9 * nr


@pytest.mark.parametrize("split", ["rowwise", "stream"])
def test_power_step_is_deterministic(split):
    n = 100_000
    A = M.c4_rows(0, n, n=n, per_row=32, seed=5)
    dev = torch.device("cuda")
    outs = []
    for _ in range(2):
        pi = PowerIteration(torch.as_tensor(A.indptr).to(dev), torch.as_tensor(A.indices).to(dev),
                            torch.as_tensor(A.data).to(dev), uniform_bounds(n, 1), 0, sched=_sched(split=split))
        pi.set_x0(torch.ones(n, dtype=torch.float64, device=dev))
        pi.iterate(5)
        outs.append(pi.x[pi.cur].cpu().numpy())
    assert np.array_equal(outs[0], outs[1])


@pytest.mark.parametrize("mode", ["store", "ce", "ce1"])
@pytest.mark.parametrize("vec", [2, 4])
@pytest.mark.parametrize("parts", [2, 3, 8])
def test_p2p_fused_step_emulated_on_one_gpu(parts, vec, mode):
    """tg_power_step_p2p_f64 with every rank's buffers on one device: per epoch the
    ranks' kernels run one after another on one stream, so each wait is already met when
    its kernel starts (nothing waits on a kernel that has not run).  Checks the pushes
    into every rank's next iterate, the slot broadcast and the epoch flags."""
    A = M.baseline_matrix("c3", scale=0.3)
    n = A.rows
    bounds = nnz_balanced_bounds(A.row_lengths(), parts)
    dev = torch.device("cuda")
    pis = []
    for r in range(parts):
        a, b = int(bounds[r]), int(bounds[r + 1])
        ip = A.indptr[a:b + 1] - A.indptr[a]
        sl = slice(int(A.indptr[a]), int(A.indptr[b]))
        pis.append(PowerIteration(torch.as_tensor(ip).to(dev), torch.as_tensor(A.indices[sl]).to(dev),
                                  torch.as_tensor(A.data[sl]).to(dev), bounds, r,
                                  sched=_sched(4, 2, 2) if vec == 2 else _sched(4, 1, 4), exchange=lambda x: None))
    assert all(p.index32 == (vec == 4) for p in pis)  # int32 indices by default with V=4
    flags = [torch.zeros(parts, dtype=torch.int64, device=dev) for _ in range(parts)]
    for pi in pis:
        pi.p2p_setup([(q.x[0], q.x[1]) for q in pis], flags)
        pi.p2p_mode = "store" if mode == "store" else "ce"
        pi.ce_chunks = 1 if mode == "ce1" else 4
    stride = pis[0].stride
    x0 = np.random.default_rng(2).uniform(-1, 1, n)
    for r, pi in enumerate(pis):
        pi.set_x0(torch.as_tensor(x0[bounds[r]:bounds[r + 1]]).to(dev))
    for r in range(parts):  # emulated all-gather of the initial shards
        src = pis[r].x[0][r * stride:(r + 1) * stride]
        for q in range(parts):
            if q != r:
                pis[q].x[0][r * stride:(r + 1) * stride].copy_(src)
    cur = 0
    iters = 9
    for _ in range(iters):
        for pi in pis:
            pi.p2p_step(cur)
        cur = 1 - cur
    for pi in pis:
        pi.cur = cur
        pi.p2p_wait()
    torch.cuda.synchronize()
    assert all(int(f.min()) == iters for f in flags)
    assert all(pi.exchange_state.epoch == iters for pi in pis)
    assert all(pi.error_word() == 0 for pi in pis)
    x = np.concatenate([pi.result()[0].cpu().numpy() for pi in pis])
    xr, nr = O.power_iteration(A, x0, iters)
    assert rel(x, xr) <= 1e-9
    assert abs(float(pis[0].result()[1]) - nr) <= 1e-9 * nr


def _single_rank_p2p(A):
    """One rank (nparts = 1) wired for the fused exchange with its own buffers and a
    zeroed flag array."""
    dev = torch.device("cuda")
    pi = PowerIteration(torch.as_tensor(A.indptr).to(dev), torch.as_tensor(A.indices).to(dev),
                        torch.as_tensor(A.data).to(dev), uniform_bounds(A.rows, 1), 0, sched=_sched(4, 2, 2),
                        exchange=lambda x: None)
    flags = [torch.zeros(1, dtype=torch.int64, device=dev)]
    pi.p2p_setup([(pi.x[0], pi.x[1])], flags)
    return pi, flags[0]


def test_p2p_step_whose_wait_runs_out_reports_it_and_the_workspace_stays_usable():
    """Failure detection of the fused exchange without a GPU fault: the step of epoch 3
    waits for a flag >= 2 that nothing sets, so its bounded device wait (2 s) runs out.
    Checks the error bit, that nothing was published, that later steps and waits return
    at once while the error word is set, and that after a restart (flags zeroed, error
    cleared) the same workspace gives the oracle's iterate (the ticket was not left
    behind by the failed launch)."""
    A = M.baseline_matrix("c3", scale=0.3)
    pi, flag = _single_rank_p2p(A)
    x0 = np.random.default_rng(9).uniform(-1, 1, A.rows)
    dev = torch.device("cuda")
    pi.set_x0(torch.as_tensor(x0).to(dev))
    torch.cuda.synchronize()
    pi.exchange_state.epoch = 2
    t0 = time.perf_counter()
    pi.p2p_step(0)  # epoch 3
    torch.cuda.synchronize()
    waited = time.perf_counter() - t0
    assert pi.error_word() == 16
    assert 1.5 <= waited < 20.0, waited
    assert int(flag.item()) == 0  # no epoch published
    t0 = time.perf_counter()
    pi.p2p_step(1)  # epoch 4: the error word is set, so no wait
    pi.p2p_wait()
    torch.cuda.synchronize()
    assert time.perf_counter() - t0 < 1.0
    assert pi.error_word() == 16 and int(flag.item()) == 0
    # restart on the same workspace
    pi.reset_exchange()
    pi.set_x0(torch.as_tensor(x0).to(dev))
    pi.iterate(6)
    x, lam = pi.result()
    assert pi.error_word() == 0 and int(flag.item()) == 6
    xr, nr = O.power_iteration(A, x0, 6)
    assert rel(x.cpu().numpy(), xr) <= 1e-9
    assert abs(float(lam) - nr) <= 1e-9 * nr


def test_p2p_wait_that_runs_out_sets_the_error_bit():
    """tg_p2p_wait for an epoch no flag reaches gives up after its 2 s bound with bit 16
    of the error word; the status of the (asynchronous) call itself is TG_OK."""
    A = M.baseline_matrix("c3", scale=0.05)
    pi, flag = _single_rank_p2p(A)
    L = lib.load()
    st = L.tg_p2p_wait(flag.data_ptr(), 1, 1, pi.ws.data_ptr(), pi.ws.numel(),
                       torch.cuda.current_stream().cuda_stream)
    assert st == lib.TG_OK
    v = ctypes.c_uint32(0)
    assert L.tg_power_error(pi.ws.data_ptr(), ctypes.byref(v), torch.cuda.current_stream().cuda_stream) == lib.TG_OK
    assert v.value == 16
    assert L.tg_power_clear_error(pi.ws.data_ptr(), torch.cuda.current_stream().cuda_stream) == lib.TG_OK
    assert pi.error_word() == 0


@pytest.mark.gpu
@pytest.mark.parametrize("parts", [1, 3, 8])
def test_renumber_columns_kernel_matches_host(parts):
    """tg_renumber_columns (device) gives the host restatement's renumbering."""
    import torch

    from tilegen_b200.power import nnz_balanced_bounds, padded_stride, renumber_columns

    rng = np.random.default_rng(parts)
    n = 10007
    row_nnz = rng.integers(0, 9, size=n)
    bounds = nnz_balanced_bounds(row_nnz, parts)
    stride = padded_stride(bounds)
    j = rng.integers(0, n, size=50001).astype(np.int64)
    want = renumber_columns(j, bounds, stride)
    got = renumber_columns(torch.as_tensor(j, device="cuda"), bounds, stride).cpu().numpy()
    assert np.array_equal(got, want)



@pytest.mark.parametrize("parts", [1, 3])
def test_int32_indices_give_the_same_iterates(parts):
    """The power step reading int32 renumbered indices (TG_FLAG_INDEX32, the default for
    the rowwise split) does the same arithmetic as with int64 ones: identical iterates."""
    A = M.baseline_matrix("c3", scale=0.3)
    bounds = nnz_balanced_bounds(A.row_lengths(), parts)
    dev = torch.device("cuda")
    x0 = np.random.default_rng(12).uniform(-1, 1, A.rows)
    outs = {}
    for i32 in (False, True):
        pis = []
        for r in range(parts):
            a, b = int(bounds[r]), int(bounds[r + 1])
            sl = slice(int(A.indptr[a]), int(A.indptr[b]))
            pis.append(PowerIteration(torch.as_tensor(A.indptr[a:b + 1] - A.indptr[a]).to(dev),
                                      torch.as_tensor(A.indices[sl]).to(dev), torch.as_tensor(A.data[sl]).to(dev),
                                      bounds, r, sched=_sched(4, 2, 2), exchange=lambda x: None, index32=i32))
        assert all(p.index32 == i32 for p in pis)
        assert all(p.indices.dtype == (torch.int32 if i32 else torch.int64) for p in pis)
        stride = pis[0].stride
        for r, pi in enumerate(pis):
            pi.set_x0(torch.as_tensor(x0[bounds[r]:bounds[r + 1]]).to(dev))
        cur = 0
        for it in range(7):
            for r in range(parts):  # emulated all-gather
                src = pis[r].x[cur][r * stride:(r + 1) * stride]
                for q in range(parts):
                    if q != r:
                        pis[q].x[cur][r * stride:(r + 1) * stride].copy_(src)
            for pi in pis:
                pi._step(pi.x[cur], pi.shard(pi.x[1 - cur]))
            cur = 1 - cur
        outs[i32] = np.concatenate([pi.x[cur][r * stride:r * stride + pi.rows].cpu().numpy()
                                    for r, pi in enumerate(pis)])
    assert np.array_equal(outs[False], outs[True])


def test_int32_renumbering_and_flag_checks():
    from tilegen_b200.power import padded_stride, renumber_columns

    rng = np.random.default_rng(5)
    n = 20011
    bounds = nnz_balanced_bounds(rng.integers(0, 9, size=n), 4)
    stride = padded_stride(bounds)
    j = rng.integers(0, n, size=70001).astype(np.int64)
    want = renumber_columns(j, bounds, stride)
    got = renumber_columns(torch.as_tensor(j, device="cuda"), bounds, stride, index32=True)
    assert got.dtype == torch.int32 and np.array_equal(got.cpu().numpy().astype(np.int64), want)
    # only the power steps take 32-bit indices
    from tilegen_b200 import device as D

    m = M.baseline_matrix("c1", scale=0.01)
    A = D.DeviceCSR.from_host(m, "cuda")
    s = lib.default_schedule()
    s.flags |= lib.TG_FLAG_INDEX32
    with pytest.raises(lib.TgError) as ei:
        D.spmv(A, torch.zeros(m.cols, dtype=torch.float64, device="cuda"), sched=s)
    assert ei.value.status == lib.TG_EUNSUPPORTED
