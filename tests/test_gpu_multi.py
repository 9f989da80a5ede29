"""The power iteration on 2+ GPUs of one node, one process per GPU (NCCL process group):
the NCCL all-gather exchange and the fused peer-memory step, against the oracle.
Skipped when fewer than two GPUs are visible."""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

N_ROWS = 300_000


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, mode, q):
    import datetime

    import torch.distributed as dist

    from tilegen_b200 import lib
    from tilegen_b200 import matrices as M
    from tilegen_b200.power import PowerIteration, uniform_bounds

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        bounds = uniform_bounds(N_ROWS, world)
        a, b = int(bounds[rank]), int(bounds[rank + 1])
        sh = M.c4_rows(a, b, n=N_ROWS, per_row=32, seed=4)
        s = lib.default_schedule()
        s.threads_per_row, s.unroll, s.vector_width, s.block_size = (4, 1, 4, 256) if mode == "p2p-v4" else (4, 2, 2, 256)
        pi = PowerIteration(torch.as_tensor(sh.indptr).to(dev), torch.as_tensor(sh.indices).to(dev),
                            torch.as_tensor(sh.data).to(dev), bounds, rank, sched=s)
        assert pi.index32 == (mode == "p2p-v4")
        if mode.startswith("p2p") or mode == "ce":
            pi.p2p_connect()
            pi.p2p_mode = "ce" if mode == "ce" else "store"
        x0 = np.random.default_rng(3).uniform(-1, 1, N_ROWS)
        res = []
        for _ in range(2):  # twice: the second solve reuses buffers, flags and epochs
            pi.set_x0(torch.as_tensor(x0[a:b]).to(dev))
            pi.iterate(15)
            x, lam = pi.result()
            torch.cuda.synchronize()
            res.append((x.cpu().numpy(), float(lam[0])))
        err = pi.error_word() if mode != "nccl" else 0
        if mode != "nccl":
            pi.close()
        q.put((rank, res, err))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("mode", ["nccl", "p2p", "p2p-v4", "ce"])
def test_power_iteration_two_gpus(mode):
    world = min(torch.cuda.device_count(), 2)
    if world < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp

    from oracle import oracle as O
    from tilegen_b200 import matrices as M

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = sorted([q.get(timeout=300) for _ in procs], key=lambda t: t[0])
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    A = M.c4_rows(0, N_ROWS, n=N_ROWS, per_row=32, seed=4)
    x0 = np.random.default_rng(3).uniform(-1, 1, N_ROWS)
    xr, nr = O.power_iteration(A, x0, 15)
    for solve in range(2):
        x = np.concatenate([o[1][solve][0] for o in out])
        assert np.abs(x - xr).max() <= 1e-9 * np.abs(xr).max()
        for o in out:
            assert abs(o[1][solve][1] - nr) <= 1e-9 * nr
    assert all(o[2] == 0 for o in out)


def _stop_worker(rank, world, port, q, stop):
    """Rank 1 stops stepping after three iterations (it stays alive, its buffers still
    mapped, nothing of it in flight); rank 0's next fused step waits for it and gives up
    after its bounded 2 s wait.  Then both ranks reset the exchange and solve again."""
    import datetime
    import time

    import torch.distributed as dist

    from tilegen_b200 import lib
    from tilegen_b200 import matrices as M
    from tilegen_b200.power import PowerIteration, uniform_bounds

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        bounds = uniform_bounds(N_ROWS, world)
        a, b = int(bounds[rank]), int(bounds[rank + 1])
        sh = M.c4_rows(a, b, n=N_ROWS, per_row=32, seed=4)
        s = lib.default_schedule()
        s.threads_per_row, s.unroll, s.vector_width, s.block_size = 4, 2, 2, 256
        pi = PowerIteration(torch.as_tensor(sh.indptr).to(dev), torch.as_tensor(sh.indices).to(dev),
                            torch.as_tensor(sh.data).to(dev), bounds, rank, sched=s)
        pi.p2p_connect()
        x0 = np.random.default_rng(3).uniform(-1, 1, N_ROWS)
        pi.set_x0(torch.as_tensor(x0[a:b]).to(dev))
        pi.iterate(3)
        torch.cuda.synchronize()
        dist.barrier()
        report = {}
        if rank == 0:
            # epoch 4 finds every flag at 3 and runs; epoch 5 waits for rank 1's flag 4,
            # which never comes
            t0 = time.perf_counter()
            pi.p2p_step(pi.cur)
            pi.p2p_step(1 - pi.cur)
            torch.cuda.synchronize()
            report["waited_s"] = time.perf_counter() - t0
            report["err"] = pi.error_word()
            t0 = time.perf_counter()
            pi.p2p_step(pi.cur)  # error word set: returns at once
            pi.p2p_wait()
            torch.cuda.synchronize()
            report["after_s"] = time.perf_counter() - t0
            stop.set()
        else:
            assert stop.wait(120)  # rank 1 does nothing until rank 0 has seen the timeout
            report["err"] = pi.error_word()
        dist.barrier()
        # restart: every rank's kernels have finished; zero the flags, clear the error
        pi.reset_exchange()
        torch.cuda.synchronize()
        dist.barrier()
        pi.set_x0(torch.as_tensor(x0[a:b]).to(dev))
        pi.iterate(15)
        x, lam = pi.result()
        torch.cuda.synchronize()
        report["err_after_restart"] = pi.error_word()
        report["x"], report["lam"] = x.cpu().numpy(), float(lam[0])
        pi.close()
        q.put((rank, report))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_p2p_peer_that_stops_is_detected_and_the_exchange_restarts():
    world = min(torch.cuda.device_count(), 2)
    if world < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp

    from oracle import oracle as O
    from tilegen_b200 import matrices as M

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    stop = ctx.Event()
    port = _free_port()
    procs = [ctx.Process(target=_stop_worker, args=(r, world, port, q, stop)) for r in range(world)]
    for p in procs:
        p.start()
    out = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    r0 = out[0]
    assert r0["err"] == 16 and 1.5 <= r0["waited_s"] < 30.0, r0
    assert r0["after_s"] < 1.0, r0
    assert out[1]["err"] == 0  # rank 1 never waited
    A = M.c4_rows(0, N_ROWS, n=N_ROWS, per_row=32, seed=4)
    x0 = np.random.default_rng(3).uniform(-1, 1, N_ROWS)
    xr, nr = O.power_iteration(A, x0, 15)
    x = np.concatenate([out[r]["x"] for r in range(world)])
    assert np.abs(x - xr).max() <= 1e-9 * np.abs(xr).max()
    assert all(abs(out[r]["lam"] - nr) <= 1e-9 * nr and out[r]["err_after_restart"] == 0 for r in range(world))
