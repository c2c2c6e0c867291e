"""tcgen05 packed GEMM (csrc/packed_gemm_tc.cu, glmvx_packed_gemm_tc) against
the CPU oracle's batched packed kernels (the reference's batch_v2 contract,
kernels/packed.vx:473ff): weights and activations split exactly into three
bf16 limbs, three kind::f16 MMAs per K step; every format, 1..64 tokens,
partial 128-row tiles, activation ranges, a non-finite token, determinism."""
import ctypes as C

import numpy as np
import pytest

from helpers import assert_close_dot, payload
from kernels.packed import LAYOUTS, unpack_for_validation

pytestmark = pytest.mark.gpu


def _device_gemm_tc(cuda_lib, kind, raw, rows, cols, x):
    from gpu.runtime import DeviceBuffer, check
    batch = x.shape[0]
    wd, xd, od = DeviceBuffer(raw.nbytes + 64), DeviceBuffer(x.nbytes + 64), DeviceBuffer(4 * batch * rows + 64)
    try:
        wd.upload(raw)
        xd.upload(x)
        check(cuda_lib, cuda_lib.glmvx_packed_gemm_tc(kind, od.ptr, wd.ptr, xd.ptr, rows, cols, batch, None),
              'gemm_tc')
        out = np.empty((batch, rows), np.float32)
        od.download(out)
        return out
    finally:
        for b in (wd, xd, od):
            b.close()


def _case(kind, rows, cols, batch, seed):
    raw = payload(kind, blocks=rows * cols // LAYOUTS[kind][0], seed=seed)
    x = np.random.default_rng(seed).normal(size=(batch, cols)).astype(np.float32)
    return raw, x


def _check(cuda_lib, oracle, kind, rows, cols, x, raw):
    got = _device_gemm_tc(cuda_lib, kind, raw, rows, cols, x)
    want = oracle.packed_linear_batch(raw, kind, (rows, cols), x)
    dec = unpack_for_validation(oracle.lib, raw, kind, (rows, cols))
    assert_close_dot(got, want, dec, x)
    return got


@pytest.mark.parametrize('kind,rows,cols,batch', [
    (8, 256, 256, 16), (8, 2048, 6144, 64), (8, 300, 4096, 9), (8, 1000, 512, 1), (8, 130, 2048, 33),
    (8, 129, 16384, 32), (12, 6144, 2048, 64), (12, 6144, 2048, 16), (12, 77, 256, 5), (12, 640, 16384, 48),
    (19, 256, 2048, 64), (19, 200, 6144, 17), (1, 128, 256, 16), (10, 128, 1024, 8), (11, 100, 2048, 24),
    (13, 260, 512, 40), (16, 128, 2048, 12), (18, 64, 2048, 20), (23, 140, 512, 63)])
def test_gemm_tc_matches_oracle(cuda_lib, oracle, kind, rows, cols, batch):
    raw, x = _case(kind, rows, cols, batch, rows + cols + batch)
    _check(cuda_lib, oracle, kind, rows, cols, x, raw)


def test_gemm_tc_activation_ranges_and_nonfinite(cuda_lib, oracle):
    """bf16 limbs keep f32's exponent range: tiny, huge and mixed chunks need
    no scaling; an infinite activation makes only its own token NaN."""
    kind, rows, cols, batch = 8, 192, 2048, 16
    raw, x = _case(kind, rows, cols, batch, 5)
    x[1] *= 1e-30
    x[2] *= 1e30
    x[3, :256] *= 1e-20
    x[3, 256:512] *= 1e20
    x[4] = 0.0
    x[6, :1024] *= 2.0 ** -140  # subnormal f32
    got = _check(cuda_lib, oracle, kind, rows, cols, x, raw)
    assert np.all(got[4] == 0.0)
    x[7, 100] = np.inf
    got = _device_gemm_tc(cuda_lib, kind, raw, rows, cols, x)
    assert np.isnan(got[7]).all()
    assert np.isfinite(np.delete(got, 7, axis=0)).all()


def test_gemm_tc_deterministic(cuda_lib):
    raw, x = _case(12, 1000, 2048, 40, 11)
    a = _device_gemm_tc(cuda_lib, 12, raw, 1000, 2048, x)
    b = _device_gemm_tc(cuda_lib, 12, raw, 1000, 2048, x)
    assert a.tobytes() == b.tobytes()


def test_gemm_tc_rejects_unsupported(cuda_lib):
    from gpu.runtime import DeviceBuffer
    buf = DeviceBuffer(1 << 20)
    try:
        # IQ1_S rows stream in 2048-column chunks; a Q6_K chunk (8 blocks of
        # 210 bytes x 128 rows) leaves no room for the tiles; 65 tokens exceed the limit
        assert cuda_lib.glmvx_packed_gemm_tc(19, buf.ptr, buf.ptr, buf.ptr, 16, 1024, 4, None) != 0
        assert cuda_lib.glmvx_packed_gemm_tc(14, buf.ptr, buf.ptr, buf.ptr, 16, 2048, 4, None) != 0
        assert cuda_lib.glmvx_packed_gemm_tc(8, buf.ptr, buf.ptr, buf.ptr, 16, 256, 65, None) != 0
    finally:
        buf.close()


@pytest.mark.parametrize('kind,cols,batch', [(8, 256, 17), (8, 512, 64), (12, 256, 40)])
def test_dispatch_takes_tc_for_many_rows(cuda_lib, oracle, kind, cols, batch):
    """glmvx_packed_gemm takes the tcgen05 GEMM (path 9) from 65536 rows and 17
    tokens (the lm_head regime); results as the oracle's."""
    from test_gpu_packed import _device_gemm
    rows = 65536 + 200  # a partial last 128-row tile
    raw, x = _case(kind, rows, cols, batch, cols + batch)
    got, path = _device_gemm(cuda_lib, kind, raw, rows, cols, x)
    assert path == 9
    want = oracle.packed_linear_batch(raw, kind, (rows, cols), x)
    dec = unpack_for_validation(oracle.lib, raw, kind, (rows, cols))
    assert_close_dot(got, want, dec, x)
