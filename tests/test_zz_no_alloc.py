"""glmvx_moe_ffn_static (scratch in a file-scope device array, no workspace
argument) against glmvx_moe_ffn (caller workspace) on the same resident layer.

The static entry is for callers that cannot allocate device memory -- a host
runtime whose allocator already owns the device's whole memory budget, or a
decode loop that must keep a fixed footprint.  Both entries run the same
kernels on the same data, so their outputs must agree byte for byte; and the
device's free memory must not change across two calls of the static entry.

Collected last on purpose: it must also pass after every other GPU test has
run in the same process (the static array is then set up on a device that has
already done other work)."""
import ctypes as C

import numpy as np
import pytest

from helpers import RTOL
from test_gpu_moe import synthetic_layer

pytestmark = pytest.mark.gpu

_P, _I32, _F32 = C.c_void_p, C.c_int32, C.c_float
STATIC_ARGS = [_P, _P, _I32, _I32, _I32, _P, _P, _I32, _I32, _F32, _I32, _P, _P, _P, _P, _P, _P, _P, _P, _P]


def _static_entry(lib):
    fn = lib.glmvx_moe_ffn_static
    fn.argtypes, fn.restype = STATIC_ARGS, _I32
    return fn


def test_static_scratch_matches_workspace_entry(gpu_backend):
    from gpu import runtime as rt
    from gpu.moe import MoELayer
    E, H, I, K, T, scale = 16, 2048, 2048, 4, 8, 2.5
    layer = synthetic_layer(E, H, I, seed=11)
    moe = MoELayer(gpu_backend, layer['router'], layer['bias'], 19, layer['gate'], layer['up'], layer['down'],
                   H, I, K, scale, shared=layer['shared'])
    lib, stream = gpu_backend.lib, gpu_backend.stream
    fn = _static_entry(lib)
    x = np.random.default_rng(5).normal(size=(T, H)).astype(np.float32)
    bufs = [rt.DeviceBuffer(n) for n in (x.nbytes, x.nbytes, 4 * T * K, 4 * T * K)]
    xd, yd, idd, wd = bufs
    try:
        xd.upload(x, stream.handle)
        moe.forward_device(yd.ptr, xd.ptr, T, idd.ptr, wd.ptr)
        want_y, want_ids, want_w = np.empty_like(x), np.empty((T, K), np.int32), np.empty((T, K), np.float32)
        stream.synchronize()
        yd.download(want_y)
        idd.download(want_ids)
        wd.download(want_w)
        def call_static():
            code = fn(yd.ptr, xd.ptr, T, H, I, moe.router_w, moe.router_bias, E, K, scale, 19, moe.gate, moe.up,
                      moe.down, *moe.shared, idd.ptr, wd.ptr, stream.handle)
            rt.check(lib, code, 'glmvx_moe_ffn_static')

        def free_bytes():
            free, total = C.c_uint64(), C.c_uint64()
            rt.check(lib, lib.glmvx_mem_get_info(C.byref(free), C.byref(total)), 'glmvx_mem_get_info')
            return free.value

        # The first call on a device looks the array's address up (which can
        # load the library's module data); measure the calls after it.
        call_static()
        stream.synchronize()
        free_before = free_bytes()
        for _ in range(2):  # two calls in a row through the same static scratch
            for b in (yd, idd, wd):
                rt.call('glmvx_memset', b.ptr, 0, b.nbytes, stream.handle)
            call_static()
            y, ids, w = np.empty_like(x), np.empty((T, K), np.int32), np.empty((T, K), np.float32)
            stream.synchronize()
            yd.download(y)
            idd.download(ids)
            wd.download(w)
            gpu_backend.device.check_device_error()
            assert ids.tolist() == want_ids.tolist()
            assert w.tobytes() == want_w.tobytes()
            assert y.tobytes() == want_y.tobytes()
            err = np.linalg.norm(y - want_y) / np.linalg.norm(want_y)
            assert err <= RTOL, err
        assert free_bytes() == free_before, 'the static entry allocated device memory'

    finally:
        stream.synchronize()
        for b in bufs:
            b.close()
        moe.close()


def test_static_scratch_rejects_oversized_layer(gpu_backend):
    """A layer whose workspace exceeds the 16 MiB array fails before any launch.

    kind 0 is also unsupported, so even a call that got past the size check
    would stop at the format check, which also precedes every launch."""
    lib = gpu_backend.lib
    fn = _static_entry(lib)
    T, H, I, E, K = 64, 6144, 2048, 256, 8
    need = lib.glmvx_moe_workspace_bytes(T, H, I, E, K, 1)
    assert need > 16 << 20
    dummy = 256  # never dereferenced: the size check precedes every launch
    code = fn(dummy, dummy, T, H, I, dummy, dummy, E, K, 2.5, 0, dummy, dummy, dummy, dummy, dummy, dummy,
              None, None, None)
    assert code == -1
    assert b'static scratch' in lib.glmvx_last_error()
