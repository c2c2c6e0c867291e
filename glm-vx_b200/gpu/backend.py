"""`vx-gpu` backend: packed GGUF projections and model primitives on a B200.

The reference GPU backend (gpu/backend.py:33-255 of gakonst/glm-vx) exposed
only expanded-f32 primitives, uploaded operands on every call, and the server
refused `--packed-weights` with it (glm_vx/server.py:147).  This backend keeps
that class's model-facing contract (matvec, rmsnorm, rope, softmax, swiglu,
route, mlp, plus layernorm/topk/index_scores/linear_batch) and adds the
packed contract of the CPU backend (kernels/backend.py:102-131):
supports_packed, packed_matvec, packed_linear_batch -- with the same
validation and ValueError wording (kernels/packed.py:45-118).

Weights live in HBM:
  * `resident(raw, kind, shape)` uploads a packed matrix once and returns a
    PackedWeight handle, accepted wherever `raw` is;
  * read-only arrays (GGUF mmap views are) are cached automatically, keyed by
    address, size, format and shape, and re-validated on every hit by a
    16-point byte fingerprint, in a byte-bounded LRU.
Activations travel through one pinned host buffer and one device arena per
backend, so a decode projection is one H2D copy, one kernel and one D2H copy
on the backend's stream.  Nothing here computes on the host; a missing
library or device raises.
"""
from collections import OrderedDict
import ctypes as C
import hashlib

import numpy as np

from . import runtime as rt
from kernels.backend import _rope_table, _rope_table_cached
from kernels.packed import LAYOUTS, _buffers, batch_input

_MAX = 2**31 - 1


def _f32(x, name='input'):
    x = np.asarray(x, dtype=np.float32)
    if x.ndim < 1 or x.size > _MAX - 1024:
        raise ValueError(name + ' must be at least one-dimensional and int32-indexable')
    return np.ascontiguousarray(x)


def _fingerprint(raw):
    n = raw.nbytes
    if n <= 256:
        return hashlib.blake2b(raw.tobytes(), digest_size=16).digest()
    step = (n - 16) // 15
    sample = b''.join(raw[i * step:i * step + 16].tobytes() for i in range(16))
    return hashlib.blake2b(sample, digest_size=16).digest()


class PackedWeight:
    """A packed matrix resident in device memory (optionally at `offset`
    inside a larger buffer it does not own)."""

    def __init__(self, buffer, kind, shape, nbytes, offset=0, owner=True):
        self.buffer, self.kind, self.shape, self.nbytes = buffer, int(kind), tuple(shape), nbytes
        self.offset, self.owner = offset, owner

    @property
    def ptr(self):
        return self.buffer.ptr + self.offset

    def close(self):
        if self.owner:
            self.buffer.close()


class GPUBackend:
    name = 'vx-gpu'

    def __init__(self, device=0, weight_cache_bytes=16 * 1024**3):
        if type(weight_cache_bytes) is not int or weight_cache_bytes < 0:
            raise ValueError('weight cache size must be nonnegative')
        self.device = rt.Device(device)
        self.lib = rt.library()
        self.stream = rt.Stream()
        self.cache = OrderedDict()  # key -> (PackedWeight, fingerprint)
        self.cache_bytes, self.cache_limit = 0, weight_cache_bytes
        self._dev = self._host = None
        self._cap = 0
        self._transient = []  # per-call uploads of writeable weights
        self._closed = False

    # ------------------------------------------------------------ plumbing
    def close(self):
        if not self._closed:
            self.stream.synchronize()
            for weight, _ in self.cache.values():
                weight.close()
            self.cache.clear()
            for b in (self._dev, self._host):
                if b is not None:
                    b.close()
            self.stream.close()
            self._closed = True

    def _begin(self):
        if self._closed:
            raise RuntimeError('GPU backend is closed')
        self.device.activate()

    def _call(self, name, *args):
        rt.check(self.lib, getattr(self.lib, name)(*args), name)

    def _reserve(self, nbytes):
        if nbytes > self._cap:
            self.stream.synchronize()
            cap = 1 << max(20, (nbytes - 1).bit_length())
            for b in (self._dev, self._host):
                if b is not None:
                    b.close()
            self._dev, self._host, self._cap = rt.DeviceBuffer(cap), rt.HostBuffer(cap), cap

    def _arena(self, input_bytes, output_bytes):
        """Offsets (256-byte aligned) of inputs then outputs in the arena,
        reserving it; no copies.  Returns (input offsets, output offsets)."""
        offsets, off = [], 0
        for nbytes in list(input_bytes) + list(output_bytes):
            offsets.append(off)
            off += (nbytes + 255) & ~255
        self._reserve(max(off, 256))
        return offsets[:len(input_bytes)], offsets[len(input_bytes):]

    def _stage(self, inputs, outputs):
        """Lay out inputs then outputs (256-byte aligned) in the arena, copy
        the inputs host->device in one transfer.  Returns device addresses of
        inputs and outputs and the output byte range."""
        offsets, off = [], 0
        for nbytes in [a.nbytes for a in inputs] + [n for n in outputs]:
            offsets.append(off)
            off += (nbytes + 255) & ~255
        self._reserve(max(off, 256))
        in_end = offsets[len(inputs)] if outputs else off
        for a, o in zip(inputs, offsets):
            if a.nbytes:
                C.memmove(self._host.ptr + o, a.ctypes.data, a.nbytes)
        if in_end:
            rt.call('glmvx_memcpy_htod', self._dev.ptr, self._host.ptr, in_end, self.stream.handle)
        ptrs = [self._dev.ptr + o for o in offsets]
        return ptrs[:len(inputs)], ptrs[len(inputs):], offsets[len(inputs):]

    def _fetch(self, out_offsets, arrays):
        """Copy outputs device->host (one transfer) and wait for the stream."""
        if out_offsets:
            lo = out_offsets[0]
            hi = out_offsets[-1] + arrays[-1].nbytes
            if hi > lo:
                rt.call('glmvx_memcpy_dtoh', self._host.ptr + lo, self._dev.ptr + lo, hi - lo, self.stream.handle)
        self.stream.synchronize()
        for o, a in zip(out_offsets, arrays):
            if a.nbytes:
                C.memmove(a.ctypes.data, self._host.ptr + o, a.nbytes)
        return arrays

    def _fetch_checked(self, out_offsets, arrays, error_offset):
        """_fetch plus the device error word, copied back in the same stream
        pass into the arena at `error_offset` (reserved by _stage): one
        synchronisation for outputs and error state; raises if a kernel
        reported an expired bounded wait."""
        if out_offsets:
            lo = out_offsets[0]
            hi = out_offsets[-1] + arrays[-1].nbytes
            if hi > lo:
                rt.call('glmvx_memcpy_dtoh', self._host.ptr + lo, self._dev.ptr + lo, hi - lo, self.stream.handle)
        rt.call('glmvx_memcpy_dtoh', self._host.ptr + error_offset, self.device.error_address(), 4, self.stream.handle)
        self.stream.synchronize()
        for o, a in zip(out_offsets, arrays):
            if a.nbytes:
                C.memmove(a.ctypes.data, self._host.ptr + o, a.nbytes)
        if C.c_int32.from_address(self._host.ptr + error_offset).value:
            self.device.check_device_error()
        return arrays

    # ----------------------------------------------------------- weights
    def unpack(self, raw, kind, blocks):
        """Decode `blocks` GGML blocks (F16: elements) of `raw` to f32 on the
        device (glmvx_unpack) and return them as a host array."""
        raw = np.ascontiguousarray(raw).view(np.uint8).reshape(-1)
        block = 1 if int(kind) == 1 else LAYOUTS[int(kind)][0]
        n = int(blocks) * block
        src, dst = rt.DeviceBuffer(max(raw.nbytes, 16)), rt.DeviceBuffer(max(4 * n, 16))
        try:
            src.upload(raw, self.stream.handle)
            rt.call('glmvx_unpack', int(kind), dst.ptr, src.ptr, int(blocks), self.stream.handle)
            out = np.empty(n, np.float32)
            dst.download(out, self.stream.handle)
            self.stream.synchronize()
            return out
        finally:
            src.close()
            dst.close()

    def resident(self, raw, kind, shape):
        """Upload a packed matrix once; the handle replaces `raw` in calls."""
        self._begin()
        _buffers(raw, kind, shape)
        buf = rt.DeviceBuffer(max(raw.nbytes, 16))
        buf.upload(raw, self.stream.handle)
        self.stream.synchronize()
        return PackedWeight(buf, kind, shape, raw.nbytes)

    def _weight(self, raw, kind, shape):
        if isinstance(raw, PackedWeight):
            if raw.kind != int(kind) or raw.shape != tuple(shape):
                raise ValueError('resident packed weight does not match kind/shape')
            return raw.ptr
        if raw.flags.writeable or raw.nbytes > self.cache_limit:
            weight = self.resident(raw, kind, shape)
            self._transient.append(weight)
            return weight.ptr
        key = (raw.ctypes.data, raw.nbytes, int(kind), tuple(shape))
        fp = _fingerprint(raw)
        hit = self.cache.get(key)
        if hit is not None:
            if hit[1] == fp:
                self.cache.move_to_end(key)
                return hit[0].ptr
            self._evict(key)
        while self.cache_bytes + raw.nbytes > self.cache_limit and self.cache:
            self._evict(next(iter(self.cache)))
        weight = self.resident(raw, kind, shape)
        self.cache[key] = (weight, fp)
        self.cache_bytes += weight.nbytes
        return weight.ptr

    def _evict(self, key):
        weight, _ = self.cache.pop(key)
        self.cache_bytes -= weight.nbytes
        weight.close()

    def _release_transient(self):
        for w in self._transient:
            w.close()
        self._transient = []

    # ----------------------------------------------------- packed contract
    def supports_packed(self, kind):
        kind = int(kind)
        return kind == 0 or kind in LAYOUTS

    def _packed_args(self, raw, kind, shape):
        if isinstance(raw, PackedWeight):
            if int(kind) != 0 and int(kind) not in LAYOUTS:
                raise ValueError('unsupported packed GGML format')
            if raw.kind != int(kind) or raw.shape != tuple(shape):
                raise ValueError('resident packed weight does not match kind/shape')
            rows, cols = raw.shape
            return rows, cols
        rows, cols, _ = _buffers(raw, kind, shape)
        return rows, cols

    def packed_matvec(self, raw, kind, shape, x):
        """out[rows] = W . x from borrowed (or resident) packed GGUF bytes."""
        rows, cols = self._packed_args(raw, kind, shape)
        x = np.asarray(x, dtype=np.float32)
        if x.ndim != 1 or x.size != cols:
            raise ValueError('packed input must match weight columns')
        if not np.isfinite(x).all():
            raise ValueError('packed input must be finite')
        out = self._packed(raw, kind, shape, np.ascontiguousarray(x)[None, :], rows, cols)[0]
        return out

    def packed_linear_batch(self, raw, kind, shape, x):
        """out[batch, rows] for up to 64 tokens from packed GGUF bytes."""
        if isinstance(raw, PackedWeight):
            rows, cols = self._packed_args(raw, kind, shape)
            x = np.asarray(x, dtype=np.float32)
            if x.ndim != 2 or x.shape[1] != cols:
                raise ValueError('packed batch input must be [batch,weight columns]')
            if len(x) > 64:
                raise ValueError('packed batch supports at most 64 tokens')
            if not np.isfinite(x).all():
                raise ValueError('packed input must be finite')
        else:
            rows, cols, _, x = batch_input(raw, kind, shape, x)
        if len(x) == 0 or rows == 0:
            return np.empty((len(x), rows), dtype=np.float32)
        return self._packed(raw, kind, shape, np.ascontiguousarray(x), rows, cols)

    def _packed(self, raw, kind, shape, x, rows, cols):
        self._begin()
        batch = x.shape[0]
        out = np.empty((batch, rows), dtype=np.float32)
        if rows == 0:
            return out
        try:
            w = self._weight(raw, kind, shape)
            (xd,), (od,), offs = self._stage([x], [out.nbytes])
            if int(kind) == 0:
                if batch == 1:
                    self._call('glmvx_matvec_f32', od, w, xd, rows, cols, self.stream.handle)
                else:
                    self._call('glmvx_matmul_nt', od, xd, w, batch, rows, cols, self.stream.handle)
            elif batch == 1:
                self._call('glmvx_packed_gemv', int(kind), od, w, xd, rows, cols, self.stream.handle)
            else:
                self._call('glmvx_packed_gemm', int(kind), od, w, xd, rows, cols, batch, self.stream.handle)
            self._fetch(offs, [out])
        finally:
            self.stream.synchronize()
            self._release_transient()
        if not np.isfinite(out).all():
            raise ValueError('nonfinite packed GGUF output')
        return out

    # --------------------------------------------------- six-op contract
    def matvec(self, w, x):
        w, x = _f32(w, 'weight'), _f32(x)
        if w.ndim != 2 or x.ndim != 1 or w.shape[1] != x.size:
            raise ValueError('matvec shape mismatch')
        raw = w.reshape(-1).view(np.uint8)
        if not w.flags.writeable:
            raw.flags.writeable = False
        return self._packed(raw, 0, w.shape, x[None, :], *w.shape)[0]

    def linear_batch(self, w, x):
        w, x = _f32(w, 'weight'), _f32(x)
        if w.ndim != 2 or x.ndim != 2 or w.shape[1] != x.shape[1]:
            raise ValueError('linear_batch expects weight[output,input] and input[batch,input]')
        raw = w.reshape(-1).view(np.uint8)
        if not w.flags.writeable:
            raw.flags.writeable = False
        if len(x) == 0 or w.shape[0] == 0:
            return np.empty((len(x), w.shape[0]), np.float32)
        out = np.empty((len(x), w.shape[0]), np.float32)
        for start in range(0, len(x), 64):  # the device batch bound is per launch
            out[start:start + 64] = self._packed(raw, 0, w.shape, x[start:start + 64], *w.shape)
        return out

    def _unary_rows(self, op, x, extra_in, tail_args):
        self._begin()
        out = np.empty_like(x)
        (xd, *rest), (od,), offs = self._stage([x, *extra_in], [out.nbytes])
        self._call(op, od, xd, *rest, *tail_args(x), self.stream.handle)
        return self._fetch(offs, [out])[0]

    def rmsnorm(self, x, w, eps):
        x, w = _f32(x), _f32(w, 'weight')
        eps = float(np.float32(eps))
        if w.ndim != 1 or w.size != x.shape[-1] or not w.size or not np.isfinite(eps) or eps <= 0:
            raise ValueError('invalid RMSNorm shape/epsilon')
        return self._unary_rows('glmvx_rmsnorm', x, [w], lambda a: (a.size // w.size, w.size, eps))

    def layernorm(self, x, w, bias, eps=1e-6):
        x, w, bias = _f32(x), _f32(w, 'weight'), _f32(bias, 'bias')
        eps = float(np.float32(eps))
        if w.ndim != 1 or bias.shape != w.shape or w.size != x.shape[-1] or not w.size or not eps > 0:
            raise ValueError('layernorm weight/bias must match the nonempty final input axis')
        return self._unary_rows('glmvx_layernorm', x, [w, bias], lambda a: (a.size // w.size, w.size, eps))

    def softmax(self, x):
        x = _f32(x)
        n = x.shape[-1]
        if not n or np.isnan(x).any() or np.isposinf(x).any() or not np.isfinite(x.reshape(-1, n)).any(axis=-1).all():
            raise ValueError('invalid softmax values')
        return self._unary_rows('glmvx_softmax', x, [], lambda a: (a.size // n, n))

    def swiglu(self, gate, up):
        gate, up = _f32(gate, 'gate'), _f32(up, 'up')
        if gate.shape != up.shape:
            raise ValueError('SwiGLU shape mismatch')
        return self._unary_rows('glmvx_swiglu', gate, [up], lambda a: (a.size,))

    def rope(self, x, position, theta):
        x = _f32(x)
        d = x.shape[-1]
        if not d or d % 2 or not np.isfinite(position) or not np.isfinite(theta) or theta <= 0:
            raise ValueError('invalid RoPE parameters')
        coefficients = _rope_table_cached if d <= 4096 else _rope_table
        cosine, sine = coefficients(d, float(position), float(theta))
        return self._unary_rows('glmvx_rope_glm', x, [cosine, sine], lambda a: (a.size // d, d))

    def route(self, logits, bias, k, scale):
        logits, bias = _f32(logits, 'logits'), _f32(bias, 'bias')
        scale = float(np.float32(scale))
        if logits.ndim != 1 or bias.shape != logits.shape or type(k) is not int or not 0 < k <= logits.size:
            raise ValueError('route expects equal one-dimensional logits and bias and 1 <= k <= experts')
        if not np.isfinite(logits).all() or not np.isfinite(bias).all() or not np.isfinite(scale):
            raise ValueError('route inputs and scale must be finite')
        self._begin()
        ids, weights = np.empty(k, np.int32), np.empty(k, np.float32)
        (ld, bd), (idd, wd), offs = self._stage([logits, bias], [ids.nbytes, weights.nbytes])
        self._call('glmvx_router', idd, wd, ld, bd, 1, logits.size, k, scale, self.stream.handle)
        return tuple(self._fetch(offs, [ids, weights]))

    def topk(self, scores, k):
        scores = _f32(scores, 'scores')
        if scores.ndim != 1 or not np.isfinite(scores).all():
            raise ValueError('topk expects finite one-dimensional scores')
        if not isinstance(k, (int, np.integer)) or not 0 <= k <= scores.size:
            raise ValueError('topk k must be an integer in [0, scores.size]')
        ids = np.empty(int(k), np.int32)
        if k == 0:
            return ids
        self._begin()
        scratch = int(self.lib.glmvx_topk_scratch_bytes(scores.size))
        (sd,), (idd, kd), offs = self._stage([scores], [ids.nbytes, max(scratch, 8)])
        self._call('glmvx_topk', idd, sd, scores.size, int(k), kd if scratch else None, self.stream.handle)
        self._fetch(offs[:1], [ids])
        return ids

    def index_scores(self, q, keys, weights, scale=None):
        q, keys, weights = [np.asarray(a, dtype=np.float32) for a in (q, keys, weights)]
        if q.ndim != 2 or keys.ndim != 2 or weights.ndim != 1:
            raise ValueError('index_scores expects query[heads,dim], keys[tokens,dim], weights[heads]')
        heads, dim = q.shape
        if heads < 1 or dim < 1 or keys.shape[1] != dim or weights.size != heads:
            raise ValueError('index_scores dimensions do not match')
        scale = float(np.float32(dim ** -0.5 if scale is None else scale))
        if not np.isfinite(scale) or any(not np.isfinite(a).all() for a in (q, keys, weights)):
            raise ValueError('index_scores inputs must be finite float32')
        tokens = keys.shape[0]
        out = np.empty(tokens, np.float32)
        if tokens == 0:
            return out
        self._begin()
        (qd, kd, wd), (od,), offs = self._stage([np.ascontiguousarray(a) for a in (q, keys, weights)], [out.nbytes])
        self._call('glmvx_index_scores', od, qd, kd, wd, tokens, heads, dim, scale, self.stream.handle)
        return self._fetch(offs, [out])[0]

    def compressed_attention(self, q_latent, q_rope, latents, rope_keys, scale):
        """Fused all-head attention over already-selected compressed KV rows,
        the contract of the reference's GPUBackend.compressed_attention
        (gpu/backend.py:233-254, used by glm_vx/model.py:209-221):
        out[h] = softmax(scale * (q_latent[h] . latents^T + q_rope[h] .
        rope_keys^T)) . latents, float32 [heads, rank]."""
        arrs = [np.ascontiguousarray(a, dtype=np.float32) for a in (q_latent, q_rope, latents, rope_keys)]
        q_latent, q_rope, latents, rope_keys = arrs
        try:
            scale = np.float32(scale)
        except (TypeError, ValueError):
            raise ValueError('MLA scale must be positive and finite') from None
        if any(a.ndim != 2 for a in arrs):
            raise ValueError('MLA expects matrices')
        heads, rank = q_latent.shape
        count, rdim = latents.shape[0], q_rope.shape[1]
        if (rank > 1024 or rdim > 128 or q_rope.shape[0] != heads or latents.shape[1] != rank
                or rope_keys.shape != (count, rdim)):
            raise ValueError('MLA shape mismatch')
        if not np.isfinite(scale) or scale <= 0:
            raise ValueError('MLA scale must be positive and finite')
        out = np.empty((heads, rank), np.float32)
        if heads == 0 or rank == 0:
            return out
        self._begin()
        need = int(self.lib.glmvx_mla_scratch_bytes(heads, rank, count))
        (qd, rd, ld, kd), (od, sd), offs = self._stage(arrs, [out.nbytes, need])
        self._call('glmvx_mla_decode', od, qd, rd, ld, kd, None, heads, rank, rdim, count, count, 0, float(scale), sd,
                   need, self.stream.handle)
        return self._fetch(offs[:1], [out])[0]

    def gemm(self, a, b, precision='f32'):
        """C = A @ B for float32 matrices A [M, K], B [K, N], the contract of
        the reference's resident GEMM (GEMMKernels.gemm, gpu/gemm.py:51-97):
        precision 'f32' multiplies and adds in f32; 'tf32_rna' rounds every
        multiplicand to TF32 (nearest, ties away from zero) and accumulates
        in f32 on the tensor cores (tcgen05, accumulators in tensor memory).
        K = 0 gives zeros."""
        if precision not in ('f32', 'tf32_rna'):
            raise ValueError("precision must be 'f32' or explicit 'tf32_rna'")
        a, b = (np.ascontiguousarray(x, dtype=np.float32) for x in (a, b))
        if a.ndim != 2 or b.ndim != 2:
            raise ValueError('A and B must be float32 matrices')
        m, k = a.shape
        if b.shape[0] != k:
            raise ValueError('GEMM inner dimensions differ')
        n = b.shape[1]
        for value, name in ((m, 'M'), (n, 'N'), (k, 'K')):
            if value >= 2 ** 31:
                raise ValueError(f'{name} must fit in int32')
        out = np.empty((m, n), np.float32)
        if m == 0 or n == 0:
            return out
        self._begin()
        (ad, bd), (od, ed), offs = self._stage([a, b], [out.nbytes, 4])
        self._call('glmvx_gemm', od, ad, bd, m, n, k, 1 if precision == 'tf32_rna' else 0, self.device.error_address(),
                   self.stream.handle)
        return self._fetch_checked(offs[:1], [out], offs[1])[0]

    @staticmethod
    def _fp8_args(weight, scales, x, batched):
        weight, scales, x = np.asarray(weight), np.asarray(scales), np.asarray(x)
        for name, arr, dtype in (('weight', weight, np.uint8), ('scales', scales, np.float32), ('x', x, np.float32)):
            if arr.dtype != dtype:
                raise ValueError(f'{name} must have dtype {np.dtype(dtype).name}')
        if weight.ndim != 2:
            raise ValueError(f'weight has incompatible shape {weight.shape}')
        rows, cols = weight.shape
        for name, value, minimum in (('rows', rows, 1), ('cols', cols, 0)):
            if not minimum <= value <= _MAX:
                raise ValueError(f'{name} must be between {minimum} and {_MAX}')
        if scales.shape != ((rows + 127) // 128, (cols + 127) // 128):
            raise ValueError(f'scales has incompatible shape {scales.shape}')
        if x.shape[-1:] != (cols,) or x.ndim != (2 if batched else 1):
            raise ValueError(f'x has incompatible shape {x.shape}')
        return tuple(np.ascontiguousarray(a) for a in (weight, scales, x))

    def fp8_matvec(self, weight, scales, x):
        """FP8 E4M3FN block-scaled projection with the contract of the
        reference's GLMKernels.fp8_matvec (gpu/runtime.py:1031-1053):
        weight uint8 [rows, cols], scales float32 [ceil(rows/128),
        ceil(cols/128)], x float32 [cols] -> float32 [rows],
        out[r] = sum_c (decode(w[r,c]) * scales[r//128, c//128]) * x[c].
        As there, non-finite inputs and the E4M3 NaN encodings are outside the
        finite-input contract and are not screened."""
        self._begin()
        weight, scales, x = self._fp8_args(weight, scales, x, False)
        rows, cols = weight.shape
        out = np.empty(rows, np.float32)
        (wd, sd, xd), (od,), offs = self._stage([weight, scales, x], [out.nbytes])
        self._call('glmvx_fp8_matvec', od, wd, sd, xd, rows, cols, self.stream.handle)
        return self._fetch(offs, [out])[0]

    def fp8_matmul(self, weight, scales, x):
        """fp8_matvec for a batch of tokens: x float32 [batch, cols] ->
        float32 [batch, rows] (row t = fp8_matvec(weight, scales, x[t])),
        through glmvx_fp8_gemm (the tcgen05 GEMM for 2..64 tokens and
        columns a multiple of 256, else one GEMV per token)."""
        self._begin()
        weight, scales, x = self._fp8_args(weight, scales, x, True)
        rows, cols = weight.shape
        out = np.empty((len(x), rows), np.float32)
        if len(x) == 0:
            return out
        (wd, sd, xd), (od,), offs = self._stage([weight, scales, x], [out.nbytes])
        self._call('glmvx_fp8_gemm', od, wd, sd, xd, rows, cols, len(x), None, self.stream.handle)
        return self._fetch(offs, [out])[0]

    def mlp(self, gate, up, down, x):
        """down(SwiGLU(gate x, up x)) on expanded f32 weights, resident intermediates."""
        gate, up, down, x = _f32(gate, 'gate weight'), _f32(up, 'up weight'), _f32(down, 'down weight'), _f32(x)
        if (gate.ndim != 2 or up.shape != gate.shape or down.ndim != 2 or x.ndim != 1
                or gate.shape[1] != x.size or down.shape[1] != gate.shape[0]):
            raise ValueError('MLP shape mismatch')
        self._begin()
        width, rows = gate.shape[0], down.shape[0]
        out = np.empty(rows, np.float32)
        ptrs = []
        try:
            for w in (gate, up, down):
                raw = w.reshape(-1).view(np.uint8)
                if not w.flags.writeable:
                    raw.flags.writeable = False
                ptrs.append(self._weight(raw, 0, w.shape))
            (xd,), (gd, ud, ad, od), offs = self._stage([x], [4 * width, 4 * width, 4 * width, out.nbytes])
            s = self.stream.handle
            self._call('glmvx_matvec_f32', gd, ptrs[0], xd, width, x.size, s)
            self._call('glmvx_matvec_f32', ud, ptrs[1], xd, width, x.size, s)
            self._call('glmvx_swiglu', ad, gd, ud, width, s)
            self._call('glmvx_matvec_f32', od, ptrs[2], ad, rows, width, s)
            self._fetch(offs[3:], [out])
        finally:
            self.stream.synchronize()
            self._release_transient()
        return out
