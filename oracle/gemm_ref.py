"""TEST INFRASTRUCTURE ONLY -- NumPy oracle for the dense GEMM contract of
the reference's resident GEMM (gpu/gemm.py:1-6, 51-97; gpu/gemm.vx:1-2,
14-73 tf32, :75ff f32).  Only tests/, smoke() and bench.py's CPU-baseline leg
may import it.

tf32_rna restates cvt.rna.tf32.f32 (the reference's "TF32
round-nearest-ties-away inputs"): the f32 bit pattern keeps its top 19 bits
(sign, 8 exponent, 10 mantissa), rounding the dropped 13 bits to nearest
with ties away from zero -- add half an ulp (0x1000) to the magnitude, then
clear the low 13 bits.  Finite inputs only, as in the reference contract.

gemm returns the float64 sum of the (rounded) products; a product of two
TF32 values is exact in f32, so the GPU result may differ from it only by
f32 accumulation rounding, which the tests bound by K * 2^-23 * (|A| @ |B|).
"""
import numpy as np


def tf32_rna(x):
    bits = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    out = ((bits + np.uint32(0x1000)) & np.uint32(0xFFFFE000)).astype(np.uint32)
    return out.view(np.float32)


def gemm(a, b, precision='f32'):
    a, b = np.asarray(a, np.float32), np.asarray(b, np.float32)
    if precision == 'tf32_rna':
        a, b = tf32_rna(a), tf32_rna(b)
    elif precision != 'f32':
        raise ValueError("precision must be 'f32' or explicit 'tf32_rna'")
    return a.astype(np.float64) @ b.astype(np.float64)


def error_bound(a, b, precision='f32'):
    """Elementwise bound on |f32-accumulated result - gemm(a, b)|."""
    a, b = np.asarray(a, np.float32), np.asarray(b, np.float32)
    if precision == 'tf32_rna':
        a, b = tf32_rna(a), tf32_rna(b)
    k = a.shape[1]
    mag = np.abs(a).astype(np.float64) @ np.abs(b).astype(np.float64)
    return (k + 2) * 2.0 ** -23 * mag + 1e-30
