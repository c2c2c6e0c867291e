"""Shared test setup.

Markers: `gpu` tests need a CUDA device (B200) and call the CUDA library
through its C ABI; everything else runs on CPU.  The oracle (oracle/) is the
checker in these tests, never the thing under test.
"""
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
PACKAGE = ROOT / 'glm-vx_b200'
for p in (str(ROOT), str(PACKAGE)):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = Path(__file__).resolve().parent / 'golden'


def pytest_configure(config):
    config.addinivalue_line('markers', 'gpu: needs a CUDA device and the sm_100a library')


@pytest.fixture(scope='session')
def golden():
    with np.load(GOLDEN / 'packed_golden.npz') as f:
        return {k: f[k] for k in f.files}


@pytest.fixture(scope='session')
def ops_golden():
    with np.load(GOLDEN / 'ops_golden.npz') as f:
        return {k: f[k] for k in f.files}


@pytest.fixture(scope='session')
def oracle():
    """VxBackend over the serial CPU oracle (the reference's numerics)."""
    from oracle import loader
    from kernels.backend import VxBackend
    return VxBackend(str(loader.serial()))


@pytest.fixture(scope='session')
def cuda_lib():
    """The sm_100a library; fails (never skips) on a GPU box without it."""
    from gpu import runtime
    if runtime.device_count() < 1:
        pytest.skip('no CUDA device')
    return runtime.library()


@pytest.fixture(scope='session')
def gpu_vx(cuda_lib):
    """VxBackend over libglmvx_cuda.so (reference ABI, host pointers)."""
    from kernels.backend import VxBackend
    from gpu.runtime import library_path
    return VxBackend(str(library_path()))


@pytest.fixture(scope='session')
def gpu_backend(cuda_lib):
    from gpu.backend import GPUBackend
    b = GPUBackend(0)
    yield b
    b.close()
