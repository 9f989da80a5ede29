"""The benchmark's gather-floor probes (libtg_gather_probe.so) gather exactly the SpMV's
x values (tg_gather_probe_f64) or the SpMM's dense rows (tg_row_gather_probe_f32); they
live outside the product library."""

from __future__ import annotations

import subprocess

import pytest

from tilegen_b200 import bench_probe, lib


@pytest.mark.gpu
@pytest.mark.parametrize("n", [0, 1, 1000, 1 << 20])
def test_gather_probe_sums_the_gathered_values(n):
    import torch

    dev = torch.device("cuda")
    g = torch.Generator(device=dev)
    g.manual_seed(5)
    x = torch.rand(1 << 16, dtype=torch.float64, device=dev, generator=g)
    idx = torch.randint(0, x.numel(), (n,), device=dev, generator=g, dtype=torch.int64)
    out = torch.zeros(1, dtype=torch.float64, device=dev)
    bench_probe.gather_probe_f64(idx.data_ptr(), n, x.data_ptr(), out.data_ptr(),
                                 torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    ref = float(x[idx].sum()) if n else 0.0
    assert abs(float(out.item()) - ref) <= 1e-9 * max(1.0, abs(ref))


@pytest.mark.gpu
@pytest.mark.parametrize("K", [64, 128])
@pytest.mark.parametrize("n", [0, 1, 1001, 1 << 18])
def test_row_gather_probe_sums_the_gathered_rows(n, K):
    """tg_row_gather_probe_f32 reads row indices[i] of B (K fp32 columns) for every i."""
    import torch

    dev = torch.device("cuda")
    g = torch.Generator(device=dev)
    g.manual_seed(6)
    B = torch.rand((1 << 14, K), dtype=torch.float32, device=dev, generator=g)
    idx = torch.randint(0, B.shape[0], (n,), device=dev, generator=g, dtype=torch.int64)
    out = torch.zeros(1, dtype=torch.float64, device=dev)
    bench_probe.row_gather_probe_f32(idx.data_ptr(), n, B.data_ptr(), K, out.data_ptr(),
                                     torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    ref = float(B.double()[idx].sum()) if n else 0.0
    assert abs(float(out.item()) - ref) <= 1e-5 * max(1.0, abs(ref))


def test_gather_probe_rejects_bad_arguments():
    L = bench_probe.load()
    assert L.tg_gather_probe_f64(None, -1, None, None, None) == lib.TG_EINVAL
    assert L.tg_gather_probe_f64(None, 5, None, None, None) == lib.TG_EINVAL
    assert L.tg_gather_probe_f64(None, 0, None, None, None) == lib.TG_OK
    assert L.tg_row_gather_probe_f32(None, 0, None, 100, None, None) == lib.TG_EINVAL  # K must be 64 or 128
    assert L.tg_row_gather_probe_f32(None, 5, None, 128, None, None) == lib.TG_EINVAL
    assert L.tg_row_gather_probe_f32(None, 0, None, 64, None, None) == lib.TG_OK


def test_probe_is_not_in_the_product_library():
    out = subprocess.run(["nm", "-D", "--defined-only", lib.lib_path()], capture_output=True, text=True).stdout
    assert "tg_gather_probe_f64" not in out and "tg_row_gather_probe_f32" not in out
