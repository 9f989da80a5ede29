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
        s.threads_per_row, s.unroll, s.vector_width, s.block_size = 4, 2, 2, 256
        pi = PowerIteration(torch.as_tensor(sh.indptr).to(dev), torch.as_tensor(sh.indices).to(dev),
                            torch.as_tensor(sh.data).to(dev), bounds, rank, sched=s)
        if mode == "p2p":
            pi.p2p_connect()
        x0 = np.random.default_rng(3).uniform(-1, 1, N_ROWS)
        res = []
        for _ in range(2):  # twice: the second solve reuses buffers, flags and epochs
            pi.set_x0(torch.as_tensor(x0[a:b]).to(dev))
            pi.iterate(15)
            x, lam = pi.result()
            torch.cuda.synchronize()
            res.append((x.cpu().numpy(), float(lam[0])))
        err = pi.error_word() if mode == "p2p" else 0
        if mode == "p2p":
            pi.close()
        q.put((rank, res, err))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("mode", ["nccl", "p2p"])
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
