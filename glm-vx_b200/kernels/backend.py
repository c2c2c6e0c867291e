"""VxBackend: the reference's model-facing kernel interface, executed by the
B200 library through the reference C ABI (host pointers).

Interface kept from the reference class (kernels/backend.py:48-237 of
gakonst/glm-vx): the method names and arguments glm_vx/model.py,
glm_vx/prefill.py and glm_vx/gguf_checkpoint.py call, the ValueError texts
their tests match, the RuntimeError when the library is missing (no
numerical fallback), and the library choice -- `library=`, else
$GLM_VX_LIBRARY, else libglmvx_cuda.so next to this package.  Each call
stages its operands on the GPU inside the library (abi_host.cu) and copies
the result back; for weights that should stay in HBM across calls use
gpu.backend.GPUBackend.

Structure: `_Abi` loads the library and binds every entry point this class
uses from a signature table spelled after include/glmvx.h; the `_need_*`
checks hold the argument rules; ops over the final axis of N-D inputs
(rmsnorm, layernorm, softmax) go through one row driver.
"""
import ctypes as C
import os
from functools import lru_cache
from pathlib import Path

import numpy as np

DEFAULT_LIBRARY = Path(__file__).resolve().parents[1] / 'libglmvx_cuda.so'
INT32_LIMIT = np.iinfo(np.int32).max

# Entry points (prefix glm_vx_) and their C parameters, one letter each:
# f = float*, i = int32*, n = int32 count, s = float scalar.
_ABI_TABLE = {
    'matvec': 'fffnn',          # out, w, x, rows, cols
    'matmul_nt': 'fffnnn',      # out, x, w, batch, rows, cols
    'rmsnorm': 'fffns',         # out, x, w, n, eps
    'layernorm': 'ffffns',      # out, x, w, bias, n, eps
    'softmax': 'ffn',           # out, x, n
    'swiglu': 'fffn',           # out, gate, up, n
    'rope_glm': 'ffffnn',       # out, x, cos, sin, rows, d
    'router': 'ifffnns',        # ids, weights, logits, bias, experts, k, scale
    'topk': 'ifnn',             # ids, scores, n, k
    'index_scores': 'ffffnnns',  # out, q, keys, w, tokens, heads, dim, scale
}
_CTYPES = {'f': C.POINTER(C.c_float), 'i': C.POINTER(C.c_int32), 'n': C.c_int32, 's': C.c_float}


class _Abi:
    """The loaded library with its entry points bound; `run` converts
    arrays to pointers and turns a nonzero status into ValueError."""

    def __init__(self, path):
        self.path = Path(path).resolve()
        try:
            self.lib = C.CDLL(str(self.path))
        except OSError as exc:
            raise RuntimeError(f'Cannot load the kernel library at {self.path}; build it with '
                               'python glm-vx_b200/build.py. No numerical fallback is enabled.') from exc
        self.fns = {}
        for op, spec in _ABI_TABLE.items():
            fn = getattr(self.lib, 'glm_vx_' + op)
            fn.argtypes, fn.restype = [_CTYPES[c] for c in spec], C.c_int32
            self.fns[op] = fn

    def run(self, op, *args):
        spec = _ABI_TABLE[op]
        conv = [a.ctypes.data_as(_CTYPES[c]) if c in 'fi' else a for c, a in zip(spec, args)]
        status = self.fns[op](*conv)
        if status:
            raise ValueError(f'Vx {op} rejected arguments (status {status})')


# ------------------------------------------------------------ argument rules
def _need_f32(value, name):
    """C-contiguous float32 copy/view with at least one axis, every extent
    (and the size) addressable with int32."""
    arr = np.ascontiguousarray(np.asarray(value, dtype=np.float32))
    if arr.ndim == 0:
        raise ValueError(f'{name} must have at least one dimension')
    if arr.size > INT32_LIMIT or max(arr.shape) > INT32_LIMIT:
        raise ValueError(f'{name} exceeds Vx int32 indexing capacity')
    return arr


def _need_eps(eps, op):
    eps = float(eps)
    if not (np.isfinite(eps) and eps > 0):
        raise ValueError(f'{op} epsilon must be finite and positive')
    return eps


def _need_row_params(x, params, op, what):
    """Per-row parameter vectors (weight, bias) matching the final axis."""
    width = x.shape[-1]
    if not width or any(p.ndim != 1 or p.size != width for p in params):
        raise ValueError(f'{op} {what} must match the nonempty final input axis')
    return width


def _rows(abi, op, x, width, params=(), scalars=()):
    """Apply a one-row entry point to every row along the final axis."""
    out = np.empty_like(x)
    src, dst = x.reshape(-1, width), out.reshape(-1, width)
    for i in range(src.shape[0]):
        abi.run(op, dst[i], src[i], *params, width, *scalars)
    return out


# ------------------------------------------------------------ RoPE tables
def _rope_table(d, position, theta):
    """cos/sin of the rotated pairs at `position`, read-only float32.  The
    arithmetic is the reference model's own (kernels/backend.py:32-39):
    float32 exponents arange(0, d, 2)/d, numpy power and cos/sin, so the
    rotated values match it bit for bit."""
    angles = position * np.power(theta, -np.arange(0, d, 2, dtype=np.float32) / d)
    table = (np.ascontiguousarray(np.cos(angles), dtype=np.float32),
             np.ascontiguousarray(np.sin(angles), dtype=np.float32))
    for t in table:
        t.flags.writeable = False
    return table


_rope_table_cached = lru_cache(maxsize=128)(_rope_table)  # used for d <= 4096: at most 2 MiB in total


class VxBackend:
    """float32 kernel backend with explicit shape and value validation."""
    name = 'vx-b200-f32'

    def __init__(self, library=None):
        self._abi = _Abi(library or os.environ.get('GLM_VX_LIBRARY') or DEFAULT_LIBRARY)
        self.library_path, self.lib = self._abi.path, self._abi.lib

    # ---------------------------------------------------------- projections
    def matvec(self, w, x):
        w, x = _need_f32(w, 'weight'), _need_f32(x, 'input')
        if not (w.ndim == 2 and x.ndim == 1 and w.shape[1] == x.size):
            raise ValueError('matvec expects weight[rows,cols] and input[cols]')
        out = np.empty(w.shape[0], np.float32)
        self._abi.run('matvec', out, w, x, w.shape[0], w.shape[1])
        return out

    def linear_batch(self, w, x):
        """x[batch, input] @ w[output, input]^T."""
        w, x = _need_f32(w, 'weight'), _need_f32(x, 'input')
        if not (w.ndim == 2 and x.ndim == 2 and w.shape[1] == x.shape[1]):
            raise ValueError('linear_batch expects weight[output,input] and input[batch,input]')
        if w.shape[0] * x.shape[0] > INT32_LIMIT:
            raise ValueError('linear_batch output exceeds Vx int32 indexing capacity')
        out = np.empty((x.shape[0], w.shape[0]), np.float32)
        self._abi.run('matmul_nt', out, x, w, x.shape[0], w.shape[0], w.shape[1])
        return out

    def supports_packed(self, kind):
        from .packed import supports
        return supports(self.lib, kind)

    @staticmethod
    def _f32_packed(raw, shape):
        """A kind-0 (F32) GGUF tensor's bytes viewed as its weight matrix."""
        return raw.view(np.float32).reshape(shape)

    @staticmethod
    def _finite_output(out):
        if not np.isfinite(out).all():
            raise ValueError('nonfinite packed GGUF output')
        return out

    def packed_matvec(self, raw, kind, shape, x):
        """Borrowed contiguous GGUF bytes times an f32 activation vector."""
        from .packed import _buffers, matvec
        if int(kind):
            return matvec(self.lib, raw, kind, shape, x)
        _buffers(raw, kind, shape)
        x = _need_f32(x, 'input')
        if not np.isfinite(x).all():
            raise ValueError('packed input must be finite')
        return self._finite_output(self.matvec(self._f32_packed(raw, shape), x))

    def packed_linear_batch(self, raw, kind, shape, x):
        """Batched projection straight from borrowed GGUF bytes."""
        from .packed import batch_input, matmul
        if int(kind):
            return matmul(self.lib, raw, kind, shape, x)
        rows, _, _, x = batch_input(raw, kind, shape, x)
        if rows == 0 or len(x) == 0:
            return np.empty((len(x), rows), np.float32)
        return self._finite_output(self.linear_batch(self._f32_packed(raw, shape), x))

    # ---------------------------------------------------- per-row primitives
    def rmsnorm(self, x, w, eps):
        x, w = _need_f32(x, 'input'), _need_f32(w, 'weight')
        width = _need_row_params(x, (w,), 'rmsnorm', 'weight')
        return _rows(self._abi, 'rmsnorm', x, width, (w,), (_need_eps(eps, 'rmsnorm'),))

    def layernorm(self, x, w, bias, eps=1e-6):
        """Affine LayerNorm along the final axis (the indexer's k_norm)."""
        x, w, bias = _need_f32(x, 'input'), _need_f32(w, 'weight'), _need_f32(bias, 'bias')
        width = _need_row_params(x, (w, bias), 'layernorm', 'weight/bias')
        return _rows(self._abi, 'layernorm', x, width, (w, bias), (_need_eps(eps, 'layernorm'),))

    def softmax(self, x):
        x = _need_f32(x, 'input')
        width = x.shape[-1]
        if not width:
            raise ValueError('softmax final axis must be nonempty')
        flat = x.reshape(-1, width)
        if np.isnan(flat).any() or np.isposinf(flat).any() or not np.isfinite(flat).any(axis=-1).all():
            raise ValueError('softmax needs one finite score per row and no NaN/+inf')
        return _rows(self._abi, 'softmax', x, width)

    # ------------------------------------------------------------ elementwise
    def swiglu(self, gate, up):
        gate, up = _need_f32(gate, 'gate'), _need_f32(up, 'up')
        if gate.shape != up.shape:
            raise ValueError('SwiGLU gate and up shapes must match')
        out = np.empty_like(gate)
        self._abi.run('swiglu', out, gate, up, gate.size)
        return out

    def rope(self, x, position, theta):
        x = _need_f32(x, 'input')
        d = x.shape[-1]
        if d == 0 or d % 2:
            raise ValueError('RoPE final dimension must be positive and even')
        position, theta = float(position), float(theta)
        if not (np.isfinite(position) and np.isfinite(theta) and theta > 0):
            raise ValueError('RoPE requires finite position and positive finite theta')
        cos, sin = (_rope_table_cached if d <= 4096 else _rope_table)(d, position, theta)
        out = np.empty_like(x)
        self._abi.run('rope_glm', out, x, cos, sin, x.size // d, d)
        return out

    # ---------------------------------------------------- routing and DSA
    def route(self, logits, bias, k, scale):
        logits, bias = _need_f32(logits, 'logits'), _need_f32(bias, 'bias')
        if logits.ndim != 1 or bias.shape != logits.shape:
            raise ValueError('route expects equal one-dimensional logits and bias')
        if not (isinstance(k, (int, np.integer)) and 0 < k <= logits.size):
            raise ValueError('route k must be an integer in [1, experts]')
        if not (np.isfinite(logits).all() and np.isfinite(bias).all() and np.isfinite(scale)):
            raise ValueError('route inputs and scale must be finite')
        ids, weights = np.empty(k, np.int32), np.empty(k, np.float32)
        self._abi.run('router', ids, weights, logits, bias, logits.size, k, float(scale))
        return ids, weights

    def topk(self, scores, k):
        """Indices of the k largest finite scores, descending, ties by the
        smaller index (int32)."""
        scores = _need_f32(scores, 'scores')
        if scores.ndim != 1 or not np.isfinite(scores).all():
            raise ValueError('topk expects finite one-dimensional scores')
        if not (isinstance(k, (int, np.integer)) and 0 <= k <= scores.size):
            raise ValueError('topk k must be an integer in [0, scores.size]')
        ids = np.empty(k, np.int32)
        self._abi.run('topk', ids, scores, scores.size, k)
        return ids

    def index_scores(self, q, keys, weights, scale=None):
        """DSA score of every cached token t: sum_h weights[h] *
        relu(dot(q[h], keys[t]) * scale)."""
        q, keys, weights = _need_f32(q, 'query'), _need_f32(keys, 'keys'), _need_f32(weights, 'weights')
        if (q.ndim, keys.ndim, weights.ndim) != (2, 2, 1):
            raise ValueError('index_scores expects query[heads,dim], keys[tokens,dim], weights[heads]')
        heads, dim = q.shape
        if 0 in (heads, dim) or keys.shape[1] != dim or weights.size != heads:
            raise ValueError('index_scores dimensions do not match')
        scale = dim ** -0.5 if scale is None else float(scale)
        if not np.isfinite(scale):
            raise ValueError('index_scores scale must be finite')
        out = np.empty(keys.shape[0], np.float32)
        self._abi.run('index_scores', out, q, keys, weights, keys.shape[0], heads, dim, scale)
        return out
