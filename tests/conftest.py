"""Shared fixtures.  `gpu` tests need a B200; everything else runs on CPU."""
import importlib
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def jx():
    return importlib.import_module("jax-rs_b200")


@pytest.fixture(scope="session")
def oracle():
    import oracle as O
    O.build()
    return O


@pytest.fixture(scope="session")
def dev(jx):
    """Initialises device 0 through the C ABI and returns a small helper."""
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    jx.init(0)
    return DeviceHelper(torch)


class DeviceHelper:
    """Moves numpy arrays to device memory (torch allocates; kernels are ours)."""

    def __init__(self, torch):
        self.torch = torch

    def put(self, a, dtype=np.float32):
        return self.torch.from_numpy(np.ascontiguousarray(a, dtype=dtype)).cuda()

    def empty(self, shape, dtype=None):
        dtype = dtype or self.torch.float32
        return self.torch.empty(shape, dtype=dtype, device="cuda")

    def full(self, shape, v):
        return self.torch.full(shape, v, dtype=self.torch.float32, device="cuda")

    def get(self, t):
        self.torch.cuda.synchronize()
        return t.cpu().numpy()

    @property
    def stream(self):
        return self.torch.cuda.current_stream().cuda_stream

    def sync(self):
        self.torch.cuda.synchronize()


def normwise_rel(got, want):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    den = np.linalg.norm(want.ravel())
    return np.linalg.norm((got - want).ravel()) / (den if den > 0 else 1.0)
