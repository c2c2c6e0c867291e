"""ctypes binding of libglmvx_cuda.so (device memory, streams, events, graphs).

Replaces the reference's ctypes CUDA Driver API runtime (gpu/runtime.py of
gakonst/glm-vx: CUDAContext :150-292, DeviceBuffer :330-380, Stream :564-600,
Event :611-663).  The native library owns every CUDA call; this module only
marshals pointers, turns nonzero status codes into exceptions, and never
falls back to host arithmetic.

The library is found at $GLM_VX_GPU_LIBRARY or next to this package
(glm-vx_b200/libglmvx_cuda.so, built by glm-vx_b200/build.py).
"""
import ctypes as C
import os
from functools import lru_cache
from pathlib import Path
from threading import RLock

import numpy as np

PACKAGE_ROOT = Path(__file__).resolve().parents[1]
DEFAULT_LIBRARY = PACKAGE_ROOT / 'libglmvx_cuda.so'

_P = C.c_void_p
_I32 = C.c_int32
_I64 = C.c_int64
_U64 = C.c_uint64
_F32 = C.c_float
_PI32 = C.POINTER(C.c_int32)
_PF32 = C.POINTER(C.c_float)

# name -> (argtypes, restype).  Every device-pointer argument is c_void_p.
SIGNATURES = {
    'glmvx_last_error': ([], C.c_char_p),
    'glmvx_version': ([], _I32),
    'glmvx_device_count': ([_PI32], _I32),
    'glmvx_set_device': ([_I32], _I32),
    'glmvx_get_device': ([_PI32], _I32),
    'glmvx_device_info': ([_I32, C.c_char_p, _I32, _PI32, _PI32, C.POINTER(_I64), C.POINTER(_I64), _PI32], _I32),
    'glmvx_malloc': ([C.POINTER(_P), _U64], _I32),
    'glmvx_free': ([_P], _I32),
    'glmvx_host_alloc': ([C.POINTER(_P), _U64], _I32),
    'glmvx_host_free': ([_P], _I32),
    'glmvx_memcpy_htod': ([_P, _P, _U64, _P], _I32),
    'glmvx_memcpy_dtoh': ([_P, _P, _U64, _P], _I32),
    'glmvx_memcpy_dtod': ([_P, _P, _U64, _P], _I32),
    'glmvx_memset': ([_P, _I32, _U64, _P], _I32),
    'glmvx_device_synchronize': ([], _I32),
    'glmvx_stream_create': ([C.POINTER(_P)], _I32),
    'glmvx_stream_destroy': ([_P], _I32),
    'glmvx_stream_synchronize': ([_P], _I32),
    'glmvx_stream_wait_event': ([_P, _P], _I32),
    'glmvx_event_create': ([C.POINTER(_P)], _I32),
    'glmvx_event_destroy': ([_P], _I32),
    'glmvx_event_record': ([_P, _P], _I32),
    'glmvx_event_synchronize': ([_P], _I32),
    'glmvx_event_elapsed_ms': ([_P, _P, _PF32], _I32),
    'glmvx_graph_begin': ([_P], _I32),
    'glmvx_graph_end': ([_P, C.POINTER(_P)], _I32),
    'glmvx_graph_launch': ([_P, _P], _I32),
    'glmvx_graph_destroy': ([_P], _I32),
    'glmvx_check_device_error': ([_PI32], _I32),
    'glmvx_device_error_address': ([C.POINTER(_P)], _I32),
    'glmvx_packed_gemv': ([_I32, _P, _P, _P, _I32, _I32, _P], _I32),
    'glmvx_packed_gemm': ([_I32, _P, _P, _P, _I32, _I32, _I32, _P], _I32),
    'glmvx_packed_gemm_path': ([_I32, _P, _P, _P, _I32, _I32, _I32, _P, _PI32], _I32),
    'glmvx_packed_gemm_tc': ([_I32, _P, _P, _P, _I32, _I32, _I32, _P], _I32),
    'glmvx_unpack': ([_I32, _P, _P, _I64, _P], _I32),
    'glmvx_matvec_f32': ([_P, _P, _P, _I32, _I32, _P], _I32),
    'glmvx_matmul_nt': ([_P, _P, _P, _I32, _I32, _I32, _P], _I32),
    'glmvx_rmsnorm': ([_P, _P, _P, _I32, _I32, _F32, _P], _I32),
    'glmvx_layernorm': ([_P, _P, _P, _P, _I32, _I32, _F32, _P], _I32),
    'glmvx_softmax': ([_P, _P, _I32, _I32, _P], _I32),
    'glmvx_swiglu': ([_P, _P, _P, _I64, _P], _I32),
    'glmvx_add': ([_P, _P, _P, _I64, _P], _I32),
    'glmvx_axpy': ([_P, _P, _F32, _I64, _P], _I32),
    'glmvx_rope_offset': ([_P, _P, _P, _P, _I32, _I32, _I32, _I32, _P], _I32),
    'glmvx_rope_glm': ([_P, _P, _P, _P, _I32, _I32, _P], _I32),
    'glmvx_router': ([_P, _P, _P, _P, _I32, _I32, _I32, _F32, _P], _I32),
    'glmvx_topk_scratch_bytes': ([_I32], _I64),
    'glmvx_topk': ([_P, _P, _I32, _I32, _P, _P], _I32),
    'glmvx_index_scores': ([_P, _P, _P, _P, _I32, _I32, _I32, _F32, _P], _I32),
    'glmvx_attention': ([_P, _P, _P, _P, _P, _P, _I32, _I32, _I32, _I32, _F32, _P, _P], _I32),
    'glmvx_mla_scratch_bytes': ([_I32, _I32, _I32], _I64),
    'glmvx_mla_decode': ([_P, _P, _P, _P, _P, _P, _I32, _I32, _I32, _I32, _I32, _I32, _F32, _P, _U64, _P], _I32),
    'glmvx_dsa_scratch_bytes': ([_I32, _I32, _I32, _I32, _I32], _I64),
    'glmvx_dsa_decode': ([_P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _I32, _I32, _I32, _I32, _I32, _I32, _I32, _I32,
                          _F32, _F32, _P, _U64, _P], _I32),
    'glmvx_dsa_decode_wait': ([_P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _I32, _I32, _I32, _I32, _I32, _I32, _I32,
                               _I32, _F32, _F32, _P, _U64, _P, _P], _I32),
    'glmvx_nonfinite_flag': ([_P, _I64, _P, _P], _I32),
    'glmvx_ipc_handle': ([_P, _P], _I32),
    'glmvx_ipc_open': ([_P, C.POINTER(C.c_void_p)], _I32),
    'glmvx_ipc_close': ([_P], _I32),
    'glmvx_gemm': ([_P, _P, _P, _I32, _I32, _I32, _I32, _P, _P], _I32),
    'glmvx_dsa_append': ([_P, _P, _P, _P, _P, _P, _P, _I32, _I32, _I32, _I32, _I32, _P, _P], _I32),
    'glmvx_moe_workspace_bytes': ([_I32, _I32, _I32, _I32, _I32, _I32], _I64),
    'glmvx_moe_ffn': ([_P, _P, _I32, _I32, _I32, _P, _P, _I32, _I32, _F32, _I32, _P, _P, _P, _P, _P, _P, _P, _U64,
                       _P, _P, _P], _I32),
    'glmvx_moe_ffn_profiled': ([_P, _P, _I32, _I32, _I32, _P, _P, _I32, _I32, _F32, _I32, _P, _P, _P, _P, _P, _P, _P,
                                _U64, _P, _P], _I32),
    'glmvx_fp8_matvec': ([_P, _P, _P, _P, _I32, _I32, _P], _I32),
    'glmvx_fp8_gemm': ([_P, _P, _P, _P, _I32, _I32, _I32, _P, _P], _I32),
    'glmvx_moe_experts': ([_P, _P, _P, _I32, _I32, _I32, _I32, _I32, _P, _P, _P, _P, _U64, _P], _I32),
    'glmvx_moe_combine': ([_P, _P, _P, _P, _P, _I32, _I32, _I32, _P], _I32),
    'glmvx_gather_rows': ([_P, _P, _P, _I32, _I32, _P], _I32),
    'glmvx_mem_get_info': ([C.POINTER(_U64), C.POINTER(_U64)], _I32),
    'glmvx_ep_create': ([C.POINTER(_P), _I32, _I32, _I32, _I32, _I32, _I32, _I32, _F32, _I32, _P, _P, _P, _P, _P,
                         _P, _P, _P], _I32),
    'glmvx_ep_mailbox': ([_P, C.POINTER(_P), C.POINTER(_U64)], _I32),
    'glmvx_ep_connect': ([_P, _P], _I32),
    'glmvx_ep_dispatch': ([_P, _P, _I32, _P, _P, _P], _I32),
    'glmvx_ep_experts': ([_P, _I32, _P], _I32),
    'glmvx_ep_combine': ([_P, _P, _I32, _P], _I32),
    'glmvx_ep_step': ([_P, _P, _P, _I32, _P, _P, _P], _I32),
    'glmvx_ep_destroy': ([_P], _I32),
    'glmvx_embed_rows': ([_P, _P, _I32, _P, _I32, _I32, _I32, _P], _I32),
    'glmvx_rope_rows': ([_P, _P, _P, _P, _P, _I32, _I32, _I32, _I32, _I64, _I32, _I32, _I64, _I32, _I32, _I32, _P],
                        _I32),
    'glmvx_rmsnorm_rows': ([_P, _P, _P, _I32, _I32, _I64, _I64, _F32, _P], _I32),
    'glmvx_absorb_query': ([_P, _P, _P, _I32, _I32, _I32, _I32, _I32, _I32, _P], _I32),
    'glmvx_absorb_value': ([_P, _P, _P, _I32, _I32, _I32, _I32, _I32, _P], _I32),
    'glmvx_scale': ([_P, _P, _F32, _I64, _P], _I32),
    'glmvx_argmax_rows': ([_P, _P, _I32, _I32, _P], _I32),
    'glmvx_fill_random': ([_P, _I32, _I64, _U64, _F32, _I32, _P], _I32),
    'glmvx_dsa_attend': ([_P, _P, _P, _P, _P, _P, _P, _I32, _I32, _I32, _I32, _I32, _I32, _F32, _P, _U64, _P], _I32),
    'glmvx_moe_job_counts': ([_I32, _I32, _I32, _I32, _I32, _I32, _P, _PI32, _P], _I32),
}


class CUDAError(RuntimeError):
    """A native call returned a nonzero status."""

    def __init__(self, operation, code, detail=''):
        self.operation, self.code, self.detail = operation, code, detail
        super().__init__(f'{operation} failed with status {code}: {detail}')


class CUDAUnavailable(RuntimeError):
    """No usable CUDA device or library; there is no CPU fallback."""


def library_path():
    return _resolved(os.environ.get('GLM_VX_GPU_LIBRARY') or str(DEFAULT_LIBRARY))


@lru_cache(maxsize=None)
def _resolved(path):
    # Resolving walks the path with one system call per component; every
    # runtime call looks the library up, so each configured path is resolved
    # once.
    return Path(path).resolve()


@lru_cache(maxsize=None)
def _load(path):
    try:
        lib = C.CDLL(str(path))
    except OSError as exc:
        raise CUDAUnavailable(f'cannot load the B200 kernel library at {path}; build it with '
                              'python glm-vx_b200/build.py. No numerical fallback is enabled.') from exc
    for name, (args, res) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes, fn.restype = args, res
    return lib


def library():
    return _load(str(library_path()))


def check(lib, code, operation):
    if code:
        raise CUDAError(operation, code, lib.glmvx_last_error().decode(errors='replace'))


def call(name, *args):
    lib = library()
    check(lib, getattr(lib, name)(*args), name)


def device_count():
    n = C.c_int32(0)
    call('glmvx_device_count', C.byref(n))
    return n.value


class Device:
    """One CUDA device: selection, properties and a lock for host-side ops."""

    def __init__(self, index=0):
        self.lib = library()
        if device_count() <= index:
            raise CUDAUnavailable(f'CUDA device {index} is not available')
        self.index = index
        self.lock = RLock()
        self.activate()
        name = C.create_string_buffer(256)
        cc, sms, smem = C.c_int32(), C.c_int32(), C.c_int32()
        l2, mem = C.c_int64(), C.c_int64()
        call('glmvx_device_info', index, name, 256, C.byref(cc), C.byref(sms), C.byref(l2), C.byref(mem),
             C.byref(smem))
        self.name = name.value.decode()
        self.compute_capability = divmod(cc.value, 10)
        self.sm_count, self.l2_bytes, self.total_memory = sms.value, l2.value, mem.value
        self.shared_memory_optin = smem.value

    def activate(self):
        call('glmvx_set_device', self.index)

    def synchronize(self):
        call('glmvx_device_synchronize')

    def error_address(self):
        """Device address of the bounded-wait error word (copy it back with a
        step's outputs; nonzero means call check_device_error)."""
        if getattr(self, '_error_address', None) is None:
            p = C.c_void_p()
            call('glmvx_device_error_address', C.byref(p))
            self._error_address = p.value
        return self._error_address

    def check_device_error(self):
        """Raise if a kernel reported an expired bounded wait since the last check."""
        code = C.c_int32(0)
        call('glmvx_check_device_error', C.byref(code))
        if code.value:
            raise CUDAError('kernel bounded wait', -3, f'device error word {code.value}')


class DeviceBuffer:
    """A device allocation; `ptr` is its address as a Python int."""

    def __init__(self, nbytes):
        self.nbytes = int(nbytes)
        p = C.c_void_p()
        call('glmvx_malloc', C.byref(p), self.nbytes)
        self.ptr = p.value or 0

    def upload(self, array, stream=None, offset=0):
        array = np.ascontiguousarray(array)
        if offset + array.nbytes > self.nbytes:
            raise ValueError('upload exceeds device buffer')
        call('glmvx_memcpy_htod', self.ptr + offset, array.ctypes.data, array.nbytes, stream)

    def download(self, array, stream=None, offset=0):
        if not array.flags.c_contiguous or offset + array.nbytes > self.nbytes:
            raise ValueError('download needs a contiguous array inside the buffer')
        call('glmvx_memcpy_dtoh', array.ctypes.data, self.ptr + offset, array.nbytes, stream)

    def close(self):
        if self.ptr:
            call('glmvx_free', self.ptr)
            self.ptr = 0

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class HostBuffer:
    """Pinned host memory with a NumPy uint8 view (`array`)."""

    def __init__(self, nbytes):
        self.nbytes = int(nbytes)
        p = C.c_void_p()
        call('glmvx_host_alloc', C.byref(p), self.nbytes)
        self.ptr = p.value or 0
        self.array = (np.ctypeslib.as_array((C.c_uint8 * self.nbytes).from_address(self.ptr))
                      if self.nbytes else np.empty(0, np.uint8))

    def view(self, dtype, count):
        return self.array[:np.dtype(dtype).itemsize * count].view(dtype)

    def close(self):
        if self.ptr:
            self.array = None
            call('glmvx_host_free', self.ptr)
            self.ptr = 0

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Stream:
    def __init__(self):
        p = C.c_void_p()
        call('glmvx_stream_create', C.byref(p))
        self.handle = p.value

    def synchronize(self):
        call('glmvx_stream_synchronize', self.handle)

    def wait_event(self, event):
        call('glmvx_stream_wait_event', self.handle, event.handle)

    def close(self):
        if self.handle:
            call('glmvx_stream_destroy', self.handle)
            self.handle = None


class Event:
    def __init__(self):
        p = C.c_void_p()
        call('glmvx_event_create', C.byref(p))
        self.handle = p.value

    def record(self, stream=None):
        call('glmvx_event_record', self.handle, stream.handle if isinstance(stream, Stream) else stream)

    def synchronize(self):
        call('glmvx_event_synchronize', self.handle)

    def elapsed_ms(self, end):
        ms = C.c_float()
        call('glmvx_event_elapsed_ms', self.handle, end.handle, C.byref(ms))
        return ms.value

    def close(self):
        if self.handle:
            call('glmvx_event_destroy', self.handle)
            self.handle = None


class Graph:
    """Capture the work issued on `stream` between begin() and end()."""

    def __init__(self, stream):
        self.stream, self.handle = stream, None

    def begin(self):
        call('glmvx_graph_begin', self.stream.handle)

    def end(self):
        p = C.c_void_p()
        call('glmvx_graph_end', self.stream.handle, C.byref(p))
        self.handle = p.value

    def launch(self):
        call('glmvx_graph_launch', self.handle, self.stream.handle)

    def close(self):
        if self.handle:
            call('glmvx_graph_destroy', self.handle)
            self.handle = None
