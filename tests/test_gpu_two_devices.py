"""One process driving two GPUs: backends on device 0 and device 1 used
alternately, each launching the kernels that raise their dynamic shared
memory limit (the int8 tensor-core GEMV, the tcgen05 packed GEMM, the FP8
tcgen05 GEMM, the tcgen05 TF32 GEMM).  The limit belongs to the kernel in
each device's context; results must match the oracle, and each other
bit for bit, on both devices."""
import numpy as np
import pytest

from helpers import assert_close_dot, payload
from kernels.packed import LAYOUTS, unpack_for_validation

pytestmark = pytest.mark.gpu


def _gpus():
    try:
        from gpu import runtime
        return runtime.device_count()
    except Exception:
        return 0


@pytest.mark.skipif(_gpus() < 2, reason='needs two GPUs')
def test_backends_on_two_devices_in_one_process(oracle):
    from gpu.backend import GPUBackend
    rng = np.random.default_rng(5)
    kind, rows, cols = 8, 65536 + 72, 512
    raw = payload(kind, blocks=rows * cols // LAYOUTS[kind][0], seed=9)
    x1 = rng.normal(size=(1, cols)).astype(np.float32)
    x40 = rng.normal(size=(40, cols)).astype(np.float32)
    w8 = rng.integers(0, 256, size=(640, 2048), dtype=np.uint8)
    w8[(w8 & 0x7F) == 0x7F] = 0x3C
    s8 = (np.abs(rng.normal(size=(5, 16))) * 0.02 + 1e-3).astype(np.float32)
    x8 = rng.normal(size=(24, 2048)).astype(np.float32)
    a = rng.normal(size=(384, 256)).astype(np.float32)
    b = rng.normal(size=(256, 512)).astype(np.float32)
    backends = [GPUBackend(0), GPUBackend(1)]
    try:
        results = [[], []]
        for _ in range(2):  # alternate: device 1's first launches come after device 0's
            for d, be in enumerate(backends):
                results[d].append((be.packed_linear_batch(raw, kind, (rows, cols), x1),
                                   be.packed_linear_batch(raw, kind, (rows, cols), x40),
                                   be.fp8_matmul(w8, s8, x8),
                                   be.gemm(a, b, 'tf32_rna')))
        for be in backends:
            be.device.check_device_error()
    finally:
        for be in backends:
            be.close()
    ref = results[0][0]
    for d in range(2):
        for got in results[d]:
            for g, r in zip(got, ref):
                assert g.tobytes() == r.tobytes()
    dec = unpack_for_validation(oracle.lib, raw, kind, (rows, cols))
    assert_close_dot(ref[0], oracle.packed_linear_batch(raw, kind, (rows, cols), x1), dec, x1)
    assert_close_dot(ref[1], oracle.packed_linear_batch(raw, kind, (rows, cols), x40), dec, x40)
    # TF32 multiplicands: each product within 2^-10 relative, f32 sums
    want = a.astype(np.float64) @ b.astype(np.float64)
    assert np.all(np.abs(ref[3] - want) <= 2.0 ** -9 * (np.abs(a).astype(np.float64) @ np.abs(b)))
