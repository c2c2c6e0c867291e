"""GPU parity for the packed codecs, GEMV and small-batch GEMM.

Every call goes through the C ABI of libglmvx_cuda.so: the reference ABI
(glm_vx_* with host pointers, via kernels.packed) or the device-pointer ABI
(glmvx_packed_*, via gpu.runtime).  Expected values come from the golden
fixtures (reference fixtures + gguf-py) and from the CPU oracle.
Decode is bit-exact; dots agree within helpers.RTOL of each row's |w||x| mass.
"""
import ctypes as C

import numpy as np
import pytest

from helpers import RTOL, assert_close_dot, payload
from kernels.packed import LAYOUTS, matmul, unpack_for_validation

pytestmark = pytest.mark.gpu
NAMES = {kind: name for kind, (_, _, name) in LAYOUTS.items()}
BATCHES = list(range(1, 18)) + [31, 32, 63, 64]


@pytest.mark.parametrize('kind', list(LAYOUTS))
def test_unpack_golden_bit_exact(gpu_vx, golden, kind):
    name = NAMES[kind]
    dec = golden[f'dec_{name}']
    got = unpack_for_validation(gpu_vx.lib, golden[f'raw_{name}'], kind, dec.shape)
    assert got.tobytes() == dec.tobytes()


@pytest.mark.parametrize('kind', list(LAYOUTS))
def test_unpack_random_blocks_bit_exact(gpu_vx, oracle, kind):
    block = LAYOUTS[kind][0]
    blocks = 4099 if block > 1 else 4099 * 8
    raw = payload(kind, blocks=blocks, seed=77 + kind)
    shape = (1, blocks * block)
    want = unpack_for_validation(oracle.lib, raw, kind, shape)
    got = unpack_for_validation(gpu_vx.lib, raw, kind, shape)
    assert got.tobytes() == want.tobytes()


def test_iq1_every_grid_index(gpu_vx, golden):
    got = unpack_for_validation(gpu_vx.lib, golden['iq1_grid_raw'], 19, (64, 256))
    assert got.tobytes() == golden['iq1_grid_dec'].tobytes()


def test_half_every_finite_pattern(gpu_vx):
    bits = np.arange(65536, dtype=np.uint16)
    bits = bits[(bits & 0x7c00) != 0x7c00]
    got = unpack_for_validation(gpu_vx.lib, bits.view(np.uint8), 1, (1, len(bits))).ravel()
    assert got.tobytes() == bits.view(np.float16).astype(np.float32).tobytes()


@pytest.mark.parametrize('kind', list(LAYOUTS))
def test_gemv_golden(gpu_vx, golden, kind):
    name = NAMES[kind]
    raw, dec = golden[f'raw_{name}'], golden[f'dec_{name}']
    for i in range(2):
        x = golden[f'x{i}_{name}']
        got = gpu_vx.packed_matvec(raw, kind, dec.shape, x)
        assert_close_dot(got, golden[f'dot{i}_{name}'], dec, x)


@pytest.mark.parametrize('kind', list(LAYOUTS))
@pytest.mark.parametrize('batch', BATCHES)
def test_batch_tiles_and_tails(gpu_vx, oracle, golden, kind, batch):
    """All codecs x batch 1..17, 31, 32, 63, 64 (tests/test_packed_batch.py:248-265)."""
    name = NAMES[kind]
    block = LAYOUTS[kind][0]
    raw, dec = golden[f'raw_{name}'], golden[f'dec_{name}']
    x = np.random.default_rng(4400 + kind + batch).normal(size=(batch, 4 * block)).astype(np.float32)
    x[:, ::2] *= np.float32(2**12)
    want = golden.get(f'bout_{name}_{batch}')
    if want is None:
        want = matmul(oracle.lib, raw, kind, dec.shape, x)
    got = gpu_vx.packed_linear_batch(raw, kind, dec.shape, x)
    assert got.shape == (batch, 3) and got.flags.c_contiguous
    assert_close_dot(got, want, dec, x)


SHAPES = [(1, 1), (3, 1), (129, 2), (1000, 8), (5, 24), (2048, 24)]  # (rows, blocks per row)


@pytest.mark.parametrize('kind', list(LAYOUTS))
@pytest.mark.parametrize('rows,nblk', SHAPES)
def test_gemv_shapes_vs_oracle(gpu_vx, oracle, kind, rows, nblk):
    block = LAYOUTS[kind][0]
    cols = nblk * (block if block > 1 else 256)
    raw = payload(kind, blocks=rows * cols // block, seed=rows * 31 + nblk)
    x = np.random.default_rng(rows + nblk).normal(size=cols).astype(np.float32)
    want = oracle.packed_matvec(raw, kind, (rows, cols), x)
    got = gpu_vx.packed_matvec(raw, kind, (rows, cols), x)
    dec = unpack_for_validation(oracle.lib, raw, kind, (rows, cols))
    assert_close_dot(got, want, dec, x)


def test_f16_odd_columns_take_the_element_path(gpu_vx, oracle):
    raw = payload(1, blocks=7 * 33, seed=5)
    x = np.random.default_rng(5).normal(size=(3, 33)).astype(np.float32)
    dec = unpack_for_validation(oracle.lib, raw, 1, (7, 33))
    assert_close_dot(gpu_vx.packed_linear_batch(raw, 1, (7, 33), x), matmul(oracle.lib, raw, 1, (7, 33), x), dec, x)
    assert_close_dot(gpu_vx.packed_matvec(raw, 1, (7, 33), x[0]), oracle.packed_matvec(raw, 1, (7, 33), x[0]), dec, x[0])


def _device_gemm(cuda_lib, kind, raw, rows, cols, x, w_offset=0):
    """Run glmvx_packed_gemm_path on device copies; returns (out, path)."""
    from gpu.runtime import DeviceBuffer, check
    batch = x.shape[0]
    wd = DeviceBuffer(raw.nbytes + 64)
    xd = DeviceBuffer(x.nbytes + 64)
    od = DeviceBuffer(4 * batch * rows + 64)
    try:
        wd.upload(raw, offset=w_offset)
        xd.upload(x)
        path = C.c_int32(-1)
        check(cuda_lib, cuda_lib.glmvx_packed_gemm_path(kind, od.ptr, wd.ptr + w_offset, xd.ptr, rows, cols, batch,
                                                        None, C.byref(path)), 'gemm')
        out = np.empty((batch, rows), np.float32)
        od.download(out)
        return out, path.value
    finally:
        for b in (wd, xd, od):
            b.close()


@pytest.mark.parametrize('kind', [8, 12, 19, 14])
def test_stream_and_generic_paths_agree(cuda_lib, oracle, kind):
    """A 16-byte aligned matrix takes the tensor-core path (Q8_0, Q4_K, IQ1_S)
    or the TMA streaming kernel (other formats); the same bytes at a 2-byte
    offset take the generic kernel.  Both match the oracle."""
    block = LAYOUTS[kind][0]
    rows, cols = 777, 2048
    raw = payload(kind, blocks=rows * cols // block, seed=kind)
    x = np.random.default_rng(kind).normal(size=(1, cols)).astype(np.float32)
    want = oracle.packed_matvec(raw, kind, (rows, cols), x[0])
    dec = unpack_for_validation(oracle.lib, raw, kind, (rows, cols))
    aligned, p1 = _device_gemm(cuda_lib, kind, raw, rows, cols, x)
    shifted, p2 = _device_gemm(cuda_lib, kind, raw, rows, cols, x, w_offset=2)
    assert (p1, p2) == ((5 if kind in (8, 12, 19) else 1), 2)
    assert_close_dot(aligned[0], want, dec, x[0])
    assert_close_dot(shifted[0], want, dec, x[0])


def test_results_are_deterministic(gpu_vx):
    raw = payload(12, blocks=6144 * 8, seed=3)
    x = np.random.default_rng(3).normal(size=2048).astype(np.float32)
    a = gpu_vx.packed_matvec(raw, 12, (6144, 2048), x)
    b = gpu_vx.packed_matvec(raw, 12, (6144, 2048), x)
    assert a.tobytes() == b.tobytes()


def _relerr(a, b):
    return float(np.linalg.norm(a.astype(np.float64) - b) / np.linalg.norm(b.astype(np.float64)))


@pytest.mark.parametrize('cfg', ['q8_0_2048x6144', 'q4_k_6144x2048', 'iq1_s_2048x6144', 'iq1_s_6144x2048'])
def test_baseline_shapes_full_size(gpu_vx, cfg):
    """BASELINE config shapes at full size, against the parallel oracle:
    strict normwise relative error <= 1e-5 on N(0,1) activations."""
    from oracle import loader
    from kernels.backend import VxBackend
    ref = VxBackend(str(loader.parallel()))
    name, shape = cfg.rsplit('_', 1)
    rows, cols = map(int, shape.split('x'))
    kind = {'q8_0': 8, 'q4_k': 12, 'iq1_s': 19}[name]
    block = LAYOUTS[kind][0]
    raw = payload(kind, blocks=rows * cols // block, seed=0)
    batches = [1, 4, 16, 64] if kind == 12 else [1]
    for batch in batches:
        x = np.random.default_rng(batch).normal(size=(batch, cols)).astype(np.float32)
        want = ref.packed_linear_batch(raw, kind, (rows, cols), x) if batch > 1 else ref.packed_matvec(raw, kind, (rows, cols), x[0])[None]
        got = gpu_vx.packed_linear_batch(raw, kind, (rows, cols), x) if batch > 1 else gpu_vx.packed_matvec(raw, kind, (rows, cols), x[0])[None]
        assert _relerr(got, want) <= RTOL, (batch, _relerr(got, want))


def test_no_kernel_reported_a_timeout(cuda_lib):
    from gpu.runtime import Device
    Device(0).check_device_error()
