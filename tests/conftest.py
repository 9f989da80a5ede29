"""pytest configuration: the `gpu` marker and shared fixtures.

Tests marked `gpu` need a CUDA device and the built libtilegen_b200.so; everything else
runs on the CPU.  GPU tests never fall back: a missing library or device is an error.
"""

from __future__ import annotations

import json
import os
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
GOLDEN = os.path.join(HERE, "golden")
if REPO not in sys.path:
    sys.path.insert(0, REPO)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200) and libtilegen_b200.so")


def load_npz(name):
    with np.load(os.path.join(GOLDEN, name), allow_pickle=False) as z:
        return {k: z[k] for k in z.files}


@pytest.fixture(scope="session")
def edge():
    return load_npz("edge257.npz")


@pytest.fixture(scope="session")
def corner():
    return load_npz("corner.npz")


@pytest.fixture(scope="session")
def kats():
    with open(os.path.join(GOLDEN, "kats.json")) as fh:
        return json.load(fh)["cases"]


@pytest.fixture(scope="session")
def corpus():
    with open(os.path.join(GOLDEN, "corpus.json")) as fh:
        return json.load(fh)


@pytest.fixture(scope="session")
def edge_csr(edge):
    from tilegen_b200.matrices import CSR

    return CSR(edge["indptr"], edge["indices"], edge["data"], tuple(int(s) for s in edge["shape"]), "edge257")


def edge_data(edge):
    """verify() inputs stored with the golden edge matrix (tilegen/verify.py:338-347)."""
    return (edge["x"], edge["w"], edge["B"], edge["U"], edge["V"], float(edge["alpha"]), float(edge["beta"]))
