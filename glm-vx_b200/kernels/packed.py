"""Host boundary for the fused packed-GGUF matvec and batch entry points.

Public surface and error behaviour follow the reference module
kernels/packed.py of gakonst/glm-vx (LAYOUTS :14-19, lookup_tables :27-37,
supports :40-42, _buffers :45-67, matvec :70-88, unpack_for_validation
:91-102, batch_input :105-118, matmul :121-155), so callers such as
glm_vx/gguf_checkpoint.py:147-151 keep working.  Checks run in the same
order and raise ValueError with the same wording.

`lib` is any ctypes library that exports the reference's C ABI
(glm_vx_packed_<fmt>, glm_vx_packed_batch_v2_<fmt>, glm_vx_unpack_<fmt>).
In this package that is libglmvx_cuda.so, whose exports run on the B200.
"""
import ctypes as C
import hashlib
import sys
from functools import lru_cache
from pathlib import Path
from typing import NamedTuple

import numpy as np

# GGML type enum -> (elements per block, bytes per block, symbol suffix).
LAYOUTS = {
    1: (1, 2, 'f16'), 8: (32, 34, 'q8_0'), 10: (256, 84, 'q2_k'), 11: (256, 110, 'q3_k'),
    12: (256, 144, 'q4_k'), 13: (256, 176, 'q5_k'), 14: (256, 210, 'q6_k'), 16: (256, 66, 'iq2_xxs'),
    18: (256, 98, 'iq3_xxs'), 19: (256, 50, 'iq1_s'), 23: (256, 136, 'iq4_xs'),
}
TABLE_SHA256 = '89c698e44735267dc93e98feb70b5a97d22351fb41440029450edba277cc11b9'
INT32_MAX = 2**31 - 1

_f32p = C.POINTER(C.c_float)
_u8p = C.POINTER(C.c_uint8)


@lru_cache(maxsize=1)
def lookup_tables():
    """(half, table): the exact fp16->f32 table and the 19,600 codebook bytes."""
    if sys.byteorder != 'little':
        raise RuntimeError('packed GGUF requires a little-endian host')
    path = Path(__file__).with_name('ggml_tables.bin')
    try:
        blob = path.read_bytes()
    except OSError as exc:
        raise RuntimeError(f'{path} is missing; run python glm-vx_b200/build.py') from exc
    if hashlib.sha256(blob).hexdigest() != TABLE_SHA256:
        raise RuntimeError('packed GGML lookup table fingerprint mismatch')
    table = np.frombuffer(blob, dtype=np.uint8)
    half = np.arange(65536, dtype=np.uint16).view(np.float16).astype(np.float32)
    half.flags.writeable = False
    return half, table


def supports(lib, kind):
    kind = int(kind)
    if kind == 0:
        return True
    return kind in LAYOUTS and hasattr(lib, 'glm_vx_packed_' + LAYOUTS[kind][2])


class _Matrix(NamedTuple):
    """A packed weight matrix's geometry after its format and shape checks."""
    rows: int
    cols: int
    suffix: str
    nbytes: int


def _matrix(kind, shape):
    """Format and shape rules (before the bytes are looked at)."""
    kind = int(kind)
    if kind != 0 and kind not in LAYOUTS:
        raise ValueError('unsupported packed GGML format')
    if len(shape) != 2 or any(type(n) is not int for n in shape):
        raise ValueError('packed weight shape must be two Python integer dimensions')
    rows, cols = shape
    block, size, suffix = (1, 4, 'f32') if kind == 0 else LAYOUTS[kind]
    if rows < 0 or cols <= 0 or cols % block:
        raise ValueError('packed matrix must have nonnegative rows and positive block-aligned cols')
    nbytes = rows * (cols // block) * size
    # The int32 ABI indexes F32 matrices by element and quantized ones by byte.
    if max(rows, cols, rows * cols) > INT32_MAX or (kind != 0 and nbytes > INT32_MAX):
        raise ValueError('packed matrix exceeds Vx int32 indexing capacity')
    return _Matrix(rows, cols, suffix, nbytes)


def _bytes_match(raw, kind, m):
    """Rules on the borrowed bytes themselves."""
    if not (isinstance(raw, np.ndarray) and raw.dtype == np.uint8 and raw.flags.c_contiguous):
        raise ValueError('packed bytes must be a contiguous uint8 array')
    if raw.nbytes != m.nbytes:
        raise ValueError('packed byte count does not match shape/format')
    if int(kind) == 0 and raw.ctypes.data % np.dtype(np.float32).alignment:
        raise ValueError('F32 packed bytes must be aligned for float loads')


def _buffers(raw, kind, shape):
    """Validate a borrowed packed matrix; returns (rows, cols, suffix)."""
    m = _matrix(kind, shape)
    _bytes_match(raw, kind, m)
    return m.rows, m.cols, m.suffix


def _status(code, what):
    if code:
        raise ValueError(f'{what} rejected arguments ({code})')


def matvec(lib, raw, kind, shape, x):
    rows, cols, suffix = _buffers(raw, kind, shape)
    x = np.asarray(x, dtype=np.float32)
    if x.ndim != 1 or x.size != cols:
        raise ValueError('packed input must match weight columns')
    if not np.isfinite(x).all():
        raise ValueError('packed input must be finite')
    x = np.ascontiguousarray(x)
    out = np.empty(rows, dtype=np.float32)
    half, table = lookup_tables()
    fn = getattr(lib, 'glm_vx_packed_' + suffix)
    fn.argtypes, fn.restype = [_f32p, _u8p, _f32p, _f32p, _u8p, C.c_int32, C.c_int32], C.c_int32
    _status(fn(out.ctypes.data_as(_f32p), raw.ctypes.data_as(_u8p), x.ctypes.data_as(_f32p),
               half.ctypes.data_as(_f32p), table.ctypes.data_as(_u8p), rows, cols), f'Vx packed {suffix}')
    if not np.isfinite(out).all():
        raise ValueError('nonfinite packed GGUF output')
    return out


def unpack_for_validation(lib, raw, kind, shape):
    """Diagnostic decode to f32; never on the serving path."""
    rows, cols, suffix = _buffers(raw, kind, shape)
    half, table = lookup_tables()
    out = np.empty(shape, dtype=np.float32)
    fn = getattr(lib, 'glm_vx_unpack_' + suffix)
    fn.argtypes, fn.restype = [_f32p, _u8p, _f32p, _u8p, C.c_int32], C.c_int32
    _status(fn(out.ctypes.data_as(_f32p), raw.ctypes.data_as(_u8p), half.ctypes.data_as(_f32p),
               table.ctypes.data_as(_u8p), rows * cols // LAYOUTS[int(kind)][0]), f'Vx unpack {suffix}')
    return out


MAX_BATCH = 64


def batch_input(raw, kind, shape, x):
    """Validate a bounded token batch before any allocation or transpose:
    returns (rows, cols, suffix, x as float32 [batch, cols])."""
    rows, cols, suffix = _buffers(raw, kind, shape)
    x = np.asarray(x, dtype=np.float32)
    if x.shape[1:] != (cols,) or x.ndim != 2:
        raise ValueError('packed batch input must be [batch,weight columns]')
    batch = len(x)
    if batch > MAX_BATCH:
        raise ValueError(f'packed batch supports at most {MAX_BATCH} tokens')
    if batch * max(cols, rows) > INT32_MAX:
        raise ValueError('packed batch exceeds Vx int32 indexing capacity')
    if not np.isfinite(x).all():
        raise ValueError('packed input must be finite')
    return rows, cols, suffix, x


def _token_tiles(x):
    """Pack [batch, cols] into consecutive transposed [cols, tile] tiles of
    64/32/16/8/4/2/1 tokens, the batch_v2 activation layout."""
    batch, cols = x.shape
    packed = np.empty(x.size, dtype=np.float32)
    token = 0
    for tile in (64, 32, 16, 8, 4, 2, 1):
        while batch - token >= tile:
            packed[token * cols:(token + tile) * cols].reshape(cols, tile)[:] = x[token:token + tile].T
            token += tile
    return packed


def matmul(lib, raw, kind, shape, x):
    """out[batch, rows]: each packed weight decoded once per token tile."""
    rows, cols, suffix, x = batch_input(raw, kind, shape, x)
    batch = len(x)
    if batch == 0 or rows == 0:
        return np.empty((batch, rows), dtype=np.float32)
    tiled = getattr(lib, 'glm_vx_packed_batch_v2_' + suffix, None)
    fn = tiled or getattr(lib, 'glm_vx_packed_batch_' + suffix, None)
    if fn is None or batch == 1:
        return np.stack([matvec(lib, raw, kind, shape, row) for row in x])
    xt = _token_tiles(x) if tiled is not None else np.ascontiguousarray(x.T)
    out = np.empty((batch, rows), dtype=np.float32)
    half, table = lookup_tables()
    fn.argtypes, fn.restype = [_f32p, _u8p, _f32p, _f32p, _u8p, C.c_int32, C.c_int32, C.c_int32], C.c_int32
    _status(fn(out.ctypes.data_as(_f32p), raw.ctypes.data_as(_u8p), xt.ctypes.data_as(_f32p),
               half.ctypes.data_as(_f32p), table.ctypes.data_as(_u8p), rows, cols, batch),
            f'Vx packed batch {suffix}')
    if not np.isfinite(out).all():
        raise ValueError('nonfinite packed GGUF output')
    return out
