"""FP8 E4M3FN block-scaled projection (gpu/fp8.vx) on the GPU against the
CPU oracle's restatement of the reference's CPU prefix (gpu/fp8.vx:3-38) and
the golden decode of all 256 encodings (gpu/test_fp8.py decode_oracle)."""
import ctypes as C

import numpy as np
import pytest

from helpers import RTOL, assert_close_dot

pytestmark = pytest.mark.gpu


def _oracle_lib():
    from oracle import loader
    lib = loader.cdll('serial')
    lib.glm_vx_fp8_matvec_reference.argtypes = [C.c_void_p] * 4 + [C.c_int32, C.c_int32]
    lib.glm_vx_fp8_matvec_reference.restype = C.c_int32
    return lib


def _want(weight, scales, x):
    lib = _oracle_lib()
    rows, cols = weight.shape
    out = np.empty(rows, np.float32)
    assert lib.glm_vx_fp8_matvec_reference(out.ctypes.data, weight.ctypes.data, scales.ctypes.data,
                                           x.ctypes.data, rows, cols) == 0
    return out


def _decoded(weight, scales, ops_golden):
    rows, cols = weight.shape
    dec = ops_golden['fp8_decode'].astype(np.float32)[weight]
    return dec * np.repeat(np.repeat(scales, 128, 0), 128, 1)[:rows, :cols]


def _case(rows, cols, seed, finite=True):
    rng = np.random.default_rng(seed)
    weight = rng.integers(0, 256, size=(rows, cols), dtype=np.uint8)
    if finite:
        weight[(weight & 0x7F) == 0x7F] = 0x3C  # keep the finite-input contract
    scales = (np.abs(rng.normal(size=((rows + 127) // 128, (cols + 127) // 128))) * 0.02 + 1e-3).astype(np.float32)
    x = rng.normal(size=cols).astype(np.float32)
    return weight, scales, x


def test_all_encodings_decode(gpu_backend, ops_golden):
    """Row r holds encoding r at column 0; x = e0 and unit scales read it back."""
    weight = np.zeros((256, 128), np.uint8)
    weight[:, 0] = np.arange(256, dtype=np.uint8)
    scales = np.ones((2, 1), np.float32)
    x = np.zeros(128, np.float32)
    x[0] = 1.0
    got = gpu_backend.fp8_matvec(weight, scales, x)
    want = ops_golden['fp8_decode'].astype(np.float32)
    nan = np.isnan(want)
    assert nan.sum() == 2 and np.isnan(got[nan]).all()
    assert np.array_equal(got[~nan], want[~nan])  # exact (the sign of zero is not kept by the row sum)


@pytest.mark.parametrize('rows,cols', [(1, 128), (7, 4), (130, 512), (300, 1000), (257, 6144), (64, 7168),
                                       (3, 13000), (5, 13001), (4100, 1024), (4097, 1040)])
def test_matvec_matches_oracle(gpu_backend, ops_golden, rows, cols):
    """Below 4096 rows four warps per row; above, one row per warp with the
    word mapping (widths a multiple of 512: 4100 x 1024, a partial last CTA)
    or 16 bytes per lane (4097 x 1040)."""
    weight, scales, x = _case(rows, cols, rows + cols)
    got = gpu_backend.fp8_matvec(weight, scales, x)
    assert_close_dot(got, _want(weight, scales, x), _decoded(weight, scales, ops_golden), x)


def test_nan_encoding_propagates(gpu_backend):
    weight, scales, x = _case(10, 256, 3)
    weight[4, 17] = 0xFF
    got = gpu_backend.fp8_matvec(weight, scales, x)
    assert np.isnan(got[4]) and np.isfinite(np.delete(got, 4)).all()


def test_device_entry_and_full_width(cuda_lib, ops_golden):
    """glmvx_fp8_matvec on device buffers at a 7168x2048 projection."""
    from gpu.runtime import DeviceBuffer, check
    weight, scales, x = _case(7168, 2048, 9)
    bufs = [DeviceBuffer(a.nbytes) for a in (weight, scales, x)] + [DeviceBuffer(4 * 7168)]
    try:
        for b, a in zip(bufs, (weight, scales, x)):
            b.upload(a)
        check(cuda_lib, cuda_lib.glmvx_fp8_matvec(bufs[3].ptr, bufs[0].ptr, bufs[1].ptr, bufs[2].ptr, 7168, 2048,
                                                   None), 'glmvx_fp8_matvec')
        got = np.empty(7168, np.float32)
        bufs[3].download(got)
    finally:
        for b in bufs:
            b.close()
    want = _want(weight, scales, x)
    assert np.linalg.norm(got - want) / np.linalg.norm(want) <= RTOL
    assert_close_dot(got, want, _decoded(weight, scales, ops_golden), x)


@pytest.mark.parametrize('change,error', [
    ({'weight': np.zeros((2, 4), np.int8)}, 'dtype uint8'),
    ({'weight': np.zeros(8, np.uint8)}, 'incompatible shape'),
    ({'weight': np.zeros((0, 4), np.uint8)}, 'rows'),
    ({'scales': np.ones((2, 1), np.float32)}, 'scales has incompatible shape'),
    ({'scales': np.ones((1, 1), np.float64)}, 'dtype float32'),
    ({'x': np.ones(5, np.float32)}, 'x has incompatible shape')])
def test_validation(gpu_backend, change, error):
    args = dict(weight=np.zeros((2, 4), np.uint8), scales=np.ones((1, 1), np.float32), x=np.ones(4, np.float32))
    args.update(change)
    with pytest.raises(ValueError, match=error):
        gpu_backend.fp8_matvec(**args)


def _device_gemm(cuda_lib, weight, scales, x):
    """glmvx_fp8_gemm on device buffers; returns (out [batch, rows], path)."""
    from gpu.runtime import DeviceBuffer, check
    rows, cols = weight.shape
    batch = x.shape[0]
    bufs = [DeviceBuffer(a.nbytes + 64) for a in (weight, scales, x)] + [DeviceBuffer(4 * batch * rows + 64)]
    path = C.c_int32(-1)
    try:
        for b, a in zip(bufs, (weight, scales, x)):
            b.upload(np.ascontiguousarray(a))
        check(cuda_lib, cuda_lib.glmvx_fp8_gemm(bufs[3].ptr, bufs[0].ptr, bufs[1].ptr, bufs[2].ptr, rows, cols, batch,
                                                 C.byref(path), None), 'glmvx_fp8_gemm')
        got = np.empty((batch, rows), np.float32)
        bufs[3].download(got)
    finally:
        for b in bufs:
            b.close()
    return got, path.value


def _want_batch(weight, scales, x):
    return np.stack([_want(weight, scales, row) for row in x])


@pytest.mark.parametrize('rows,cols,batch', [(128, 256, 2), (300, 6144, 16), (1000, 2048, 64), (7168, 2048, 33),
                                             (77, 512, 5), (2048, 6144, 24), (129, 16384, 48)])
def test_gemm_tc_matches_oracle(cuda_lib, ops_golden, rows, cols, batch):
    """The tcgen05 path (cols a multiple of 256, 2..64 tokens): every token's
    row as the reference's matvec within the f32 dot-product bound."""
    weight, scales, _ = _case(rows, cols, rows + cols + batch)
    x = np.random.default_rng(batch).normal(size=(batch, cols)).astype(np.float32)
    got, path = _device_gemm(cuda_lib, weight, scales, x)
    assert path == 9
    assert_close_dot(got, _want_batch(weight, scales, x), _decoded(weight, scales, ops_golden), x)


@pytest.mark.parametrize('rows,cols,batch', [(130, 1000, 8), (64, 256, 1), (9, 13001, 3)])
def test_gemm_falls_back_to_matvec(cuda_lib, ops_golden, rows, cols, batch):
    weight, scales, _ = _case(rows, cols, rows + cols)
    x = np.random.default_rng(batch).normal(size=(batch, cols)).astype(np.float32)
    got, path = _device_gemm(cuda_lib, weight, scales, x)
    assert path == 1
    want = _want_batch(weight, scales, x)
    dec = _decoded(weight, scales, ops_golden)
    for t in range(batch):
        assert np.array_equal(got[t], _device_gemm(cuda_lib, weight, scales, x[t:t + 1])[0][0])
        assert_close_dot(got[t], want[t], dec, x[t])


def test_gemm_tc_all_encodings_exact(cuda_lib, ops_golden):
    """Row r holds encoding r at column 0: with unit scales and x = e0 every
    token reads the decoded value back exactly (the limb split is exact); the
    two NaN encodings make only their own rows NaN."""
    weight = np.zeros((256, 256), np.uint8)
    weight[:, 0] = np.arange(256, dtype=np.uint8)
    scales = np.ones((2, 2), np.float32)
    x = np.zeros((4, 256), np.float32)
    x[:, 0] = [1.0, -2.0, 0.5, 2.0 ** -20]
    got, path = _device_gemm(cuda_lib, weight, scales, x)
    assert path == 9
    want = ops_golden['fp8_decode'].astype(np.float32)
    nan = np.isnan(want)
    for t in range(4):
        assert np.isnan(got[t][nan]).all()
        assert np.array_equal(got[t][~nan], want[~nan] * x[t, 0])


def test_gemm_tc_scale_tiles(cuda_lib, ops_golden):
    """Each 128 x 128 tile takes its own scale: scales spanning 2^-30 .. 2^30
    and a zero tile."""
    rows, cols, batch = 384, 1024, 12
    weight, _, _ = _case(rows, cols, 21)
    rng = np.random.default_rng(4)
    scales = (2.0 ** rng.integers(-30, 31, size=(3, 8))).astype(np.float32)
    scales[1, 5] = 0.0
    x = rng.normal(size=(batch, cols)).astype(np.float32)
    got, path = _device_gemm(cuda_lib, weight, scales, x)
    assert path == 9
    assert_close_dot(got, _want_batch(weight, scales, x), _decoded(weight, scales, ops_golden), x)


def test_gemm_tc_deterministic_and_backend(cuda_lib, gpu_backend, ops_golden):
    weight, scales, _ = _case(640, 2048, 8)
    x = np.random.default_rng(8).normal(size=(20, 2048)).astype(np.float32)
    a, _ = _device_gemm(cuda_lib, weight, scales, x)
    b, _ = _device_gemm(cuda_lib, weight, scales, x)
    assert a.tobytes() == b.tobytes()
    assert np.array_equal(gpu_backend.fp8_matmul(weight, scales, x), a)
    assert gpu_backend.fp8_matmul(weight, scales, x[:0]).shape == (0, 640)
    with pytest.raises(ValueError, match='x has incompatible shape'):
        gpu_backend.fp8_matmul(weight, scales, x[0])
