"""Tensor-core (int8 mma) packed GEMV/GEMM path against the CPU oracle.

The path multiplies the GGML block integers by the activations split into
four exact int8 limbs per 256-column chunk; these tests pin it to the
reference's f32 semantics (kernels/packed.vx:154-470 and the batch_v2
forms) on shapes, batches and activation ranges that stress the limb
scaling, and check which kernel ran."""
import ctypes as C

import numpy as np
import pytest

from helpers import assert_close_dot, payload
from kernels.packed import LAYOUTS, matmul, unpack_for_validation

pytestmark = pytest.mark.gpu

KINDS = [8, 12, 19]
PATH_MMA = 5


def _gemm(cuda_lib, kind, raw, rows, cols, x):
    """glmvx_packed_gemm_path on device copies -> (out [batch, rows], path)."""
    from gpu.runtime import DeviceBuffer, check
    batch = x.shape[0]
    wd, xd, od = DeviceBuffer(raw.nbytes + 64), DeviceBuffer(x.nbytes + 64), DeviceBuffer(4 * batch * rows + 64)
    try:
        wd.upload(raw)
        xd.upload(np.ascontiguousarray(x, np.float32))
        path = C.c_int32(-1)
        check(cuda_lib, cuda_lib.glmvx_packed_gemm_path(kind, od.ptr, wd.ptr, xd.ptr, rows, cols, batch, None,
                                                        C.byref(path)), 'glmvx_packed_gemm_path')
        out = np.empty((batch, rows), np.float32)
        od.download(out)
        return out, path.value
    finally:
        for b in (wd, xd, od):
            b.close()


PATH_GEMM = 6


def _batch_path(kind, cols, batch):
    """Tensor-core path taken for an aligned matrix: the f16 GEMM for 8..64
    tokens of Q4_K, Q8_0 and IQ1_S (IQ1_S rows of 2048-column multiples), the
    int8 GEMV kernel otherwise."""
    gemm = 8 <= batch <= 64 and cols % 256 == 0 and (kind in (8, 12) or (kind == 19 and cols % 2048 == 0))
    return PATH_GEMM if gemm else PATH_MMA


def _want(oracle, raw, kind, rows, cols, x):
    if x.shape[0] == 1:
        return oracle.packed_matvec(raw, kind, (rows, cols), x[0])[None]
    return matmul(oracle.lib, raw, kind, (rows, cols), x)


@pytest.mark.parametrize('kind', KINDS)
@pytest.mark.parametrize('rows,cols', [(777, 512), (130, 1024), (61, 1536), (300, 2048), (17, 3072), (40, 6144),
                                       (9, 8192)])
@pytest.mark.parametrize('batch', [1, 2, 3, 8])
def test_mma_matches_oracle(cuda_lib, oracle, kind, rows, cols, batch):
    block = LAYOUTS[kind][0]
    raw = payload(kind, blocks=rows * cols // block, seed=rows + cols + kind)
    x = np.random.default_rng(batch * 7 + cols).normal(size=(batch, cols)).astype(np.float32)
    got, path = _gemm(cuda_lib, kind, raw, rows, cols, x)
    # IQ1_S rows are whole 16-byte units only when cols % 2048 == 0; other
    # widths keep the CUDA-core kernels.  Eight or more tokens of Q4_K and
    # IQ1_S take the f16 GEMM (test_gpu_gemm.py).
    if kind != 19 or cols % 2048 == 0:
        assert path == _batch_path(kind, cols, batch)
    else:
        assert path not in (PATH_MMA, PATH_GEMM)
    dec = unpack_for_validation(oracle.lib, raw, kind, (rows, cols))
    want = _want(oracle, raw, kind, rows, cols, x)
    for t in range(batch):
        assert_close_dot(got[t], want[t], dec, x[t])


@pytest.mark.parametrize('kind', KINDS)
@pytest.mark.parametrize('batch', [5, 16, 33, 64])
def test_mma_batches(cuda_lib, oracle, kind, batch):
    rows, cols = 96, 2048
    block = LAYOUTS[kind][0]
    raw = payload(kind, blocks=rows * cols // block, seed=batch)
    x = np.random.default_rng(batch).normal(size=(batch, cols)).astype(np.float32)
    got, path = _gemm(cuda_lib, kind, raw, rows, cols, x)
    assert path == _batch_path(kind, cols, batch)
    dec = unpack_for_validation(oracle.lib, raw, kind, (rows, cols))
    want = _want(oracle, raw, kind, rows, cols, x)
    for t in range(batch):
        assert_close_dot(got[t], want[t], dec, x[t])


def _activation_cases(cols, rng):
    base = rng.normal(size=cols).astype(np.float32)
    outlier = base.copy()
    outlier[::97] *= 3000.0  # a few channels far above the rest of their chunk
    zeros = base.copy()
    zeros[256:768] = 0.0     # whole chunks of zeros
    tiny = (base * np.float32(1e-30)).astype(np.float32)
    huge = (base * np.float32(1e30)).astype(np.float32)
    decades = np.repeat(np.float32(10.0) ** rng.integers(-20, 20, size=cols // 256), 256).astype(np.float32)
    ones = np.ones(cols, np.float32)
    return dict(outlier=outlier, zeros=zeros, tiny=tiny, huge=huge, decades=(base * decades).astype(np.float32),
                ones=ones)


@pytest.mark.parametrize('kind', KINDS)
def test_mma_activation_ranges(cuda_lib, oracle, kind):
    """Per-chunk power-of-two scaling keeps the f32 tolerance for outlier
    channels, zero chunks, tiny and huge magnitudes, and chunk scales spread
    over 40 decades."""
    rows, cols = 64, 2048
    block = LAYOUTS[kind][0]
    raw = payload(kind, blocks=rows * cols // block, seed=11)
    dec = unpack_for_validation(oracle.lib, raw, kind, (rows, cols))
    cases = _activation_cases(cols, np.random.default_rng(2))
    x = np.stack(list(cases.values()))
    got, path = _gemm(cuda_lib, kind, raw, rows, cols, x)
    assert path == PATH_MMA
    want = _want(oracle, raw, kind, rows, cols, x)
    for t, name in enumerate(cases):
        assert np.isfinite(got[t]).all(), name
        assert_close_dot(got[t], want[t], dec, x[t])


@pytest.mark.parametrize('kind', KINDS)
def test_mma_nonfinite_activation_gives_nonfinite_rows(cuda_lib, kind):
    """The device ABI does not validate activations; a non-finite value must
    not turn into a finite result (the Python boundary rejects it earlier)."""
    rows, cols = 32, 2048
    block = LAYOUTS[kind][0]
    raw = payload(kind, blocks=rows * cols // block, seed=3)
    x = np.random.default_rng(3).normal(size=(2, cols)).astype(np.float32)
    x[0, 300] = np.inf
    x[1, 5] = np.nan
    got, path = _gemm(cuda_lib, kind, raw, rows, cols, x)
    assert path == PATH_MMA
    assert not np.isfinite(got).any()


@pytest.mark.parametrize('kind', KINDS)
def test_mma_is_deterministic(cuda_lib, kind):
    rows, cols = 1000, 6144
    block = LAYOUTS[kind][0]
    raw = payload(kind, blocks=rows * cols // block, seed=4)
    x = np.random.default_rng(4).normal(size=(3, cols)).astype(np.float32)
    a, _ = _gemm(cuda_lib, kind, raw, rows, cols, x)
    b, _ = _gemm(cuda_lib, kind, raw, rows, cols, x)
    assert a.tobytes() == b.tobytes()


def test_mma_two_tokens_share_a_job_independently(cuda_lib):
    """Token 1 of a job must not leak into token 0: batch 2 equals two batch-1 calls."""
    rows, cols, kind = 200, 2048, 19
    raw = payload(kind, blocks=rows * cols // 256, seed=8)
    x = np.random.default_rng(8).normal(size=(2, cols)).astype(np.float32)
    x[1] *= 1000.0
    both, _ = _gemm(cuda_lib, kind, raw, rows, cols, x)
    one, _ = _gemm(cuda_lib, kind, raw, rows, cols, x[:1])
    two, _ = _gemm(cuda_lib, kind, raw, rows, cols, x[1:])
    assert both[0].tobytes() == one[0].tobytes()
    assert both[1].tobytes() == two[0].tobytes()
