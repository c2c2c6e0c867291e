"""The GEMM oracle's TF32 rounding against hand-computed cases
(cvt.rna.tf32.f32: nearest, ties away from zero; gpu/gemm.vx:1-2)."""
import numpy as np

from oracle import gemm_ref


def test_tf32_rna_ties_away_and_nearest():
    one = np.float32(1.0)
    half_ulp = np.float32(2.0 ** -11)  # TF32 keeps 10 mantissa bits: ulp(1) = 2^-10
    cases = [(one + half_ulp, 1 + 2.0 ** -10),                       # tie -> away from zero
             (-(one + half_ulp), -(1 + 2.0 ** -10)),
             (np.float32(1 + 2.0 ** -11 - 2.0 ** -23), 1.0),           # below the tie -> down
             (np.float32(1 + 3 * 2.0 ** -11), 1 + 2 * 2.0 ** -10),     # tie 1.5 ulp -> 2 ulp (away, not even)
             (np.float32(3.0), 3.0), (np.float32(0.0), 0.0)]
    for x, want in cases:
        assert float(gemm_ref.tf32_rna(np.array([x]))[0]) == want, (x, want)


def test_gemm_ref_shapes_and_bound():
    rng = np.random.default_rng(0)
    a, b = rng.normal(size=(5, 7)).astype(np.float32), rng.normal(size=(7, 3)).astype(np.float32)
    c = gemm_ref.gemm(a, b, 'tf32_rna')
    assert c.shape == (5, 3)
    assert np.all(np.abs(c - gemm_ref.gemm(a, b)) < 7 * 2.0 ** -9 * (np.abs(a) @ np.abs(b)))
    assert gemm_ref.gemm(np.zeros((2, 0), np.float32), np.zeros((0, 3), np.float32)).shape == (2, 3)
