"""Dense GEMM drop-in (csrc/gemm.cu glmvx_gemm, GPUBackend.gemm) against the
reference contract (gpu/gemm.py:51-97): tf32_rna on tcgen05 tensor cores and
f32 on CUDA cores, ragged shapes, K = 0, the TF32 rounding of single products
(exact: a product of two TF32 values is exact in f32) and argument errors."""
import numpy as np
import pytest

from oracle import gemm_ref

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize('precision', ['tf32_rna', 'f32'])
@pytest.mark.parametrize('m,n,k', [(1, 1, 1), (16, 8, 8), (129, 130, 33), (128, 128, 64), (300, 257, 1000),
                                   (1024, 1024, 1024), (7, 300, 4097)])
def test_gemm_matches_oracle(gpu_backend, precision, m, n, k):
    rng = np.random.default_rng(m * 7 + n * 3 + k)
    a = rng.normal(size=(m, k)).astype(np.float32)
    b = rng.normal(size=(k, n)).astype(np.float32)
    got = gpu_backend.gemm(a, b, precision)
    want = gemm_ref.gemm(a, b, precision)
    assert got.shape == (m, n) and got.dtype == np.float32
    assert np.all(np.abs(got - want) <= gemm_ref.error_bound(a, b, precision))
    if precision == 'tf32_rna' and k >= 64:  # the rounding is really applied
        assert np.abs(got - gemm_ref.gemm(a, b, 'f32')).max() > np.abs(got - want).max()


def test_tf32_single_products_exact(gpu_backend):
    """K = 1: C = rna(a) * rna(b) exactly, with operands on and off the
    rounding ties (ties go away from zero, not to even, not truncated)."""
    base = np.float32(1.0) + np.float32(2.0 ** -11) * np.arange(-8, 8, dtype=np.float32)
    a = np.concatenate([base, -base, base * np.float32(3.7)]).astype(np.float32)[:, None]
    b = np.concatenate([base[::-1], base * np.float32(-0.3)]).astype(np.float32)[None, :]
    got = gpu_backend.gemm(a, b, 'tf32_rna')
    want = (gemm_ref.tf32_rna(a).astype(np.float64) @ gemm_ref.tf32_rna(b).astype(np.float64)).astype(np.float32)
    assert np.array_equal(got, want)


def test_gemm_edges(gpu_backend):
    a, b = np.ones((3, 0), np.float32), np.ones((0, 5), np.float32)
    for p in ('f32', 'tf32_rna'):
        assert np.array_equal(gpu_backend.gemm(a, b, p), np.zeros((3, 5), np.float32))
        assert gpu_backend.gemm(np.ones((0, 4), np.float32), np.ones((4, 2), np.float32), p).shape == (0, 2)
    with pytest.raises(ValueError, match='inner dimensions'):
        gpu_backend.gemm(np.ones((2, 3), np.float32), np.ones((4, 2), np.float32))
    with pytest.raises(ValueError, match='precision'):
        gpu_backend.gemm(np.ones((2, 3), np.float32), np.ones((3, 2), np.float32), 'tf32')
