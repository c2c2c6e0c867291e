"""The `vx-gpu` backend's packed contract: same validation as the CPU
boundary, results within tolerance of the oracle, device weight cache."""
import numpy as np
import pytest

from helpers import assert_close_dot, payload
from kernels.packed import LAYOUTS, unpack_for_validation

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize('kind', list(LAYOUTS))
def test_packed_matvec_and_batch(gpu_backend, oracle, kind):
    block = LAYOUTS[kind][0]
    rows, cols = 300, 2 * (block if block > 1 else 256)
    raw = payload(kind, blocks=rows * cols // block, seed=kind + 100)
    dec = unpack_for_validation(oracle.lib, raw, kind, (rows, cols))
    x = np.random.default_rng(kind).normal(size=(5, cols)).astype(np.float32)
    assert_close_dot(gpu_backend.packed_matvec(raw, kind, (rows, cols), x[0]),
                     oracle.packed_matvec(raw, kind, (rows, cols), x[0]), dec, x[0])
    assert_close_dot(gpu_backend.packed_linear_batch(raw, kind, (rows, cols), x),
                     oracle.packed_linear_batch(raw, kind, (rows, cols), x), dec, x)


def test_f32_kind_zero(gpu_backend, oracle):
    w = np.random.default_rng(2).normal(size=(33, 70)).astype(np.float32)
    x = np.random.default_rng(3).normal(size=(4, 70)).astype(np.float32)
    raw = w.view(np.uint8).reshape(-1)
    np.testing.assert_allclose(gpu_backend.packed_matvec(raw, 0, w.shape, x[0]), oracle.packed_matvec(raw, 0, w.shape, x[0]),
                               rtol=3e-5, atol=3e-5)
    np.testing.assert_allclose(gpu_backend.packed_linear_batch(raw, 0, w.shape, x),
                               oracle.packed_linear_batch(raw, 0, w.shape, x), rtol=3e-5, atol=3e-5)


def test_read_only_weights_are_cached_and_fingerprinted(gpu_backend):
    raw = payload(19, blocks=64 * 8, seed=1).reshape(-1).copy()
    raw.flags.writeable = False
    x = np.ones(2048, np.float32)
    before = len(gpu_backend.cache)
    a = gpu_backend.packed_matvec(raw, 19, (64, 2048), x)
    b = gpu_backend.packed_matvec(raw, 19, (64, 2048), x)
    assert len(gpu_backend.cache) == before + 1 and a.tobytes() == b.tobytes()
    writable = raw.copy()  # writeable arrays are uploaded per call, never cached
    gpu_backend.packed_matvec(writable, 19, (64, 2048), x)
    assert len(gpu_backend.cache) == before + 1


def test_resident_handle(gpu_backend, oracle):
    raw = payload(8, blocks=128 * 64, seed=4)
    handle = gpu_backend.resident(raw, 8, (128, 2048))
    x = np.random.default_rng(4).normal(size=2048).astype(np.float32)
    dec = unpack_for_validation(oracle.lib, raw, 8, (128, 2048))
    assert_close_dot(gpu_backend.packed_matvec(handle, 8, (128, 2048), x), oracle.packed_matvec(raw, 8, (128, 2048), x),
                     dec, x)
    with pytest.raises(ValueError, match='kind/shape'):
        gpu_backend.packed_matvec(handle, 8, (64, 4096), np.ones(4096, np.float32))
    handle.close()


@pytest.mark.parametrize('change,error', [
    ({'raw': np.zeros(49, np.uint8)}, 'byte count'), ({'raw': np.zeros(50, np.float32)}, 'uint8'),
    ({'raw': np.zeros(100, np.uint8)[::2]}, 'contiguous'), ({'shape': (1, 255)}, 'block-aligned'),
    ({'shape': (-1, 256)}, 'nonnegative'), ({'shape': (2**31, 256)}, 'int32'), ({'shape': (1, 0)}, 'positive'),
    ({'shape': (True, 256)}, 'integer'), ({'kind': 999}, 'unsupported'),
    ({'x': np.ones(255, np.float32)}, 'columns'), ({'x': np.full(256, np.nan, np.float32)}, 'finite')])
def test_same_errors_as_cpu_boundary(gpu_backend, change, error):
    args = dict(raw=np.zeros(50, np.uint8), kind=19, shape=(1, 256), x=np.ones(256, np.float32))
    args.update(change)
    with pytest.raises(ValueError, match=error):
        gpu_backend.packed_matvec(**args)


def test_nonfinite_output_rejected(gpu_backend):
    raw = np.zeros(50, np.uint8)
    raw[:2] = np.frombuffer(np.float16(np.inf).tobytes(), np.uint8)
    with pytest.raises(ValueError, match='nonfinite'):
        gpu_backend.packed_matvec(raw, 19, (1, 256), np.ones(256, np.float32))


def test_empty_shapes(gpu_backend):
    assert gpu_backend.packed_linear_batch(np.zeros(0, np.uint8), 19, (0, 256), np.zeros((7, 256), np.float32)).shape == (7, 0)
    assert gpu_backend.packed_linear_batch(np.zeros(50, np.uint8), 19, (1, 256), np.zeros((0, 256), np.float32)).shape == (0, 1)
    assert gpu_backend.packed_matvec(np.zeros(0, np.uint8), 8, (0, 32), np.ones(32, np.float32)).shape == (0,)
