"""f16 tensor-core GEMM for token batches (csrc/packed_gemm.cu, path 6)
against the CPU oracle's batched packed kernels (the reference's batch_v2
contract, kernels/packed.vx:473ff): Q4_K, IQ1_S and Q8_0 at 8..64 tokens, shapes
with one and several row tiles and column slices, ragged row counts,
activation ranges far from N(0,1), a non-finite token, determinism."""
import numpy as np
import pytest

from helpers import RTOL, assert_close_dot, payload
from kernels.packed import LAYOUTS, unpack_for_validation
from test_gpu_packed import _device_gemm

pytestmark = pytest.mark.gpu

PATH_GEMM = 6
PATH_TC = 9


def _case(kind, rows, cols, batch, seed):
    raw = payload(kind, blocks=rows * cols // LAYOUTS[kind][0], seed=seed)
    x = np.random.default_rng(seed).normal(size=(batch, cols)).astype(np.float32)
    return raw, x


@pytest.mark.parametrize('kind,rows,cols,batch', [
    (12, 6144, 2048, 16), (12, 6144, 2048, 64), (12, 300, 4096, 9), (12, 16, 256, 8), (12, 777, 2048, 33),
    (12, 2048, 6144, 24), (19, 2048, 6144, 32), (19, 6144, 2048, 8), (19, 130, 2048, 64), (19, 4100, 4096, 12),
    (8, 2048, 6144, 16), (8, 2048, 6144, 64), (8, 300, 4096, 9), (8, 1000, 256, 8), (8, 4099, 2048, 40),
    (8, 200, 8192, 8), (12, 640, 16384, 64), (12, 100, 16384, 13)])
def test_gemm_matches_oracle(cuda_lib, oracle, kind, rows, cols, batch):
    raw, x = _case(kind, rows, cols, batch, rows + batch)
    got, path = _device_gemm(cuda_lib, kind, raw, rows, cols, x)
    # long rows at 33..64 tokens take the tcgen05 GEMM (path 9, its own tests
    # in test_gpu_packed_tc.py); the rest the f16 GEMM
    long_rows = cols >= (12288 if kind == 19 else 6144)
    assert path == (PATH_TC if batch > 32 and (long_rows or rows >= 16384) else PATH_GEMM)
    want = oracle.packed_linear_batch(raw, kind, (rows, cols), x)
    dec = unpack_for_validation(oracle.lib, raw, kind, (rows, cols))
    assert_close_dot(got, want, dec, x)


@pytest.mark.parametrize('kind', [12, 19, 8])
def test_gemm_activation_ranges(cuda_lib, oracle, kind):
    """Each token's chunks are scaled separately: tiny, huge, mixed and zero
    chunks keep the relative accuracy of the others."""
    rows, cols, batch = 96, 2048, 12
    raw, x = _case(kind, rows, cols, batch, 5)
    x[1] *= 1e-30
    x[2] *= 1e30
    x[3, :256] *= 1e-20
    x[3, 256:512] *= 1e20
    x[4] = 0.0
    x[5, ::7] = 0.0
    x[6, :1024] *= 2.0 ** -140  # subnormal f32 chunks
    got, path = _device_gemm(cuda_lib, kind, raw, rows, cols, x)
    assert path == PATH_GEMM
    want = oracle.packed_linear_batch(raw, kind, (rows, cols), x)
    dec = unpack_for_validation(oracle.lib, raw, kind, (rows, cols))
    assert np.all(got[4] == 0.0)
    assert_close_dot(got, want, dec, x)


@pytest.mark.parametrize('kind', [12, 19, 8])
def test_gemm_nonfinite_token(cuda_lib, kind):
    """A non-finite activation makes that token's outputs NaN and leaves the
    other tokens finite."""
    rows, cols, batch = 64, 2048, 8
    raw, x = _case(kind, rows, cols, batch, 7)
    x[3, 100] = np.inf
    got, path = _device_gemm(cuda_lib, kind, raw, rows, cols, x)
    assert path == PATH_GEMM
    assert np.isnan(got[3]).all()
    assert np.isfinite(np.delete(got, 3, axis=0)).all()


def test_gemm_deterministic_and_matches_gemv_path(cuda_lib, oracle):
    """Same bytes twice give the same bits; 7 tokens (the int8 path) and 8
    tokens (this path) agree with the oracle alike."""
    kind, rows, cols = 12, 1000, 2048
    raw, x = _case(kind, rows, cols, 8, 11)
    a, _ = _device_gemm(cuda_lib, kind, raw, rows, cols, x)
    b, _ = _device_gemm(cuda_lib, kind, raw, rows, cols, x)
    assert a.tobytes() == b.tobytes()
    seven, p7 = _device_gemm(cuda_lib, kind, raw, rows, cols, x[:7])
    assert p7 == 5
    want = oracle.packed_linear_batch(raw, kind, (rows, cols), x)
    dec = unpack_for_validation(oracle.lib, raw, kind, (rows, cols))
    assert_close_dot(a, want, dec, x)
    assert_close_dot(seven, want[:7], dec, x[:7])


def test_gemm_full_size_normwise(gpu_vx):
    """Config-1 shape at 64 tokens: strict normwise error against the parallel oracle."""
    from oracle import loader
    from kernels.backend import VxBackend
    ref = VxBackend(str(loader.parallel()))
    raw, x = _case(12, 6144, 2048, 64, 0)
    got = gpu_vx.packed_linear_batch(raw, 12, (6144, 2048), x)
    want = ref.packed_linear_batch(raw, 12, (6144, 2048), x)
    err = np.linalg.norm(got.astype(np.float64) - want) / np.linalg.norm(want.astype(np.float64))
    assert err <= RTOL, err


@pytest.mark.parametrize('kind,rows,cols,batch,path', [
    (8, 512, 16384, 1, 7), (8, 300, 16384, 2, 7), (8, 6144, 16384, 1, 7), (8, 700, 16384, 16, 8),
    (8, 130, 24576, 8, 8), (12, 256, 16384, 1, 7), (12, 100, 32768, 3, 7), (19, 256, 16384, 1, 7),
    (19, 96, 65536, 9, 8)])
def test_long_rows_in_column_segments(cuda_lib, oracle, kind, rows, cols, batch, path):
    """Rows too long for one tensor-core plan (config 3's Q8_0 o_proj reads
    16384 columns) run as equal column segments, later ones adding onto the
    output in segment order; same tolerance against the oracle as one pass."""
    raw, x = _case(kind, rows, cols, batch, rows + cols + batch)
    got, p = _device_gemm(cuda_lib, kind, raw, rows, cols, x)
    assert p == path
    want = oracle.packed_linear_batch(raw, kind, (rows, cols), x)
    dec = unpack_for_validation(oracle.lib, raw, kind, (rows, cols))
    assert_close_dot(got, want, dec, x)
    again, _ = _device_gemm(cuda_lib, kind, raw, rows, cols, x)
    assert again.tobytes() == got.tobytes()
