"""The multi-rank host logic of the power iteration on CPU: 2 `gloo` ranks, each with
its nnz-balanced shard, renumbered columns and the padded all-gather layout; the local
step is a host implementation of the tg_power_step_f64 contract (the GPU kernel is
covered by tests/test_gpu_power.py)."""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import oracle as O
from tilegen_b200 import matrices as M
from tilegen_b200.power import PowerIteration, nnz_balanced_bounds, padded_stride, renumber_columns


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _matrix():
    return M.baseline_matrix("c3", scale=0.02)


def _worker(rank, world, port, iters, out_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        A = _matrix()
        bounds = nnz_balanced_bounds(A.row_lengths(), world)
        a, b = int(bounds[rank]), int(bounds[rank + 1])
        ip = torch.as_tensor(A.indptr[a:b + 1] - A.indptr[a])
        sl = slice(int(A.indptr[a]), int(A.indptr[b]))
        ix = torch.as_tensor(A.indices[sl])
        dv = torch.as_tensor(A.data[sl])
        holder = {}

        def step(x_full, y_shard):
            # the tg_power_step_f64 contract on the host
            pi = holder["pi"]
            slots = x_full.view(pi.parts, pi.stride)[:, -1]
            s = 1.0 / float(np.sqrt(slots.sum().item()))
            local = (pi.indptr.numpy(), pi.indices.numpy(), pi.data.numpy())
            y = O.spmv(local, x_full.numpy()) * s
            y_shard[:pi.rows] = torch.as_tensor(y)
            y_shard[-1] = float(np.dot(y, y))

        def norm2(shard):
            shard[-1] = float((shard[:-1] ** 2).sum())

        def finalize(x_full, x_out, lam_out):
            pi = holder["pi"]
            nrm = float(np.sqrt(x_full.view(pi.parts, pi.stride)[:, -1].sum().item()))
            x_out.copy_(pi.shard(x_full)[:pi.rows] / nrm)
            lam_out.fill_(nrm)

        def exchange(x_full):
            pi = holder["pi"]
            parts = list(x_full.view(pi.parts, pi.stride).unbind(0))
            dist.all_gather(parts, pi.shard(x_full).clone())

        pi = PowerIteration(ip, ix, dv, bounds, rank, step=step, norm2=norm2, finalize=finalize, exchange=exchange)
        holder["pi"] = pi
        x0 = np.random.default_rng(4).uniform(-1, 1, A.rows)
        pi.set_x0(torch.as_tensor(x0[a:b]))
        pi.iterate(iters)
        x, lam = pi.result()
        out_q.put((rank, x.numpy(), float(lam[0])))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_match_oracle_power_iteration():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    iters = 6
    procs = [ctx.Process(target=_worker, args=(r, 2, port, iters, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted([q.get(timeout=120) for _ in procs])
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    A = _matrix()
    x = np.concatenate([r[1] for r in res])
    x0 = np.random.default_rng(4).uniform(-1, 1, A.rows)
    xr, nr = O.power_iteration(A, x0, iters)
    assert np.abs(x - xr).max() <= 1e-12 * np.abs(xr).max() + 1e-15
    assert abs(res[0][2] - nr) <= 1e-12 * nr and res[0][2] == res[1][2]


def test_bounds_stride_and_renumbering():
    L = np.array([5, 0, 0, 7, 1, 1, 1, 20, 0, 3])
    b = nnz_balanced_bounds(L, 3)
    assert b[0] == 0 and b[-1] == L.size and np.all(np.diff(b) >= 0)
    nnz_per = [L[b[r]:b[r + 1]].sum() for r in range(3)]
    assert max(nnz_per) <= L.sum()  # every nonzero assigned once
    assert sum(nnz_per) == L.sum()
    stride = padded_stride(b)
    assert stride % 32 == 0 and stride >= np.diff(b).max() + 1
    j = np.arange(L.size)
    jr = renumber_columns(j, b, stride)
    owner = np.searchsorted(b, j, side="right") - 1
    assert np.array_equal(jr, owner * stride + j - b[owner])
    assert np.array_equal(renumber_columns(torch.as_tensor(j), b, stride).numpy(), jr)
