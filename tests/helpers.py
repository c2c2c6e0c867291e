"""Numerical helpers shared by the parity tests."""
import hashlib

import numpy as np

from kernels.packed import LAYOUTS

# The one tolerance for every f32 packed GEMV/GEMM parity check.  The
# reference sums each row sequentially; the GPU sums in a tree with FMA.  Both
# are within a few f32 ulps of the exact sum, so the check is relative to the
# row's absolute mass sum_j |w_j x_j| (cancellation-safe) plus a normwise bound.
RTOL = 1e-5


def payload(kind, blocks=12, seed=None):
    """Random raw blocks with finite fp16 scales (the reference fixture shape:
    scale slots per format as in tests/test_packed_matvec.py:40-44)."""
    block, size, name = LAYOUTS[kind]
    rng = np.random.default_rng(934 + kind if seed is None else seed)
    raw = rng.integers(0, 256, size=(blocks, size), dtype=np.uint8)
    positions = {'q2_k': [80, 82], 'q3_k': [108], 'q6_k': [208], 'q4_k': [0, 2], 'q5_k': [0, 2]}.get(name, [0])
    scales = (np.abs(rng.normal(size=blocks)) * 0.01).astype(np.float16)
    for p in positions:
        raw[:, p:p + 2] = scales.view(np.uint8).reshape(-1, 2)
    if kind == 1:
        raw = rng.normal(size=blocks).astype(np.float16).view(np.uint8).reshape(blocks, 2)
    return raw


def assert_close_dot(actual, expected, weights, x, rtol=RTOL):
    """|y - y_ref| <= rtol * sum_j |w_j x_j| per element, and normwise."""
    actual = np.asarray(actual, np.float64)
    expected = np.asarray(expected, np.float64)
    w = np.asarray(weights, np.float64)
    x = np.asarray(x, np.float64)
    mass = np.abs(x) @ np.abs(w).T if x.ndim == 2 else np.abs(w) @ np.abs(x)
    err = np.abs(actual - expected)
    bad = err > rtol * mass + 1e-30
    assert not bad.any(), f'{bad.sum()} outputs exceed {rtol} x row mass; worst {np.max(err / (mass + 1e-30))}'
    norm = np.linalg.norm(expected)
    if norm > 0:
        assert np.linalg.norm(actual - expected) <= rtol * max(norm, np.linalg.norm(mass)), 'normwise error'


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).digest()
