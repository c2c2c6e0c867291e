"""Resident DSA decode attention for a batch of requests on one B200.

The reference keeps each request's compressed cache as Python lists of
NumPy rows (`RequestCache`, glm_vx/model.py:176-181 latents and rope keys,
:146-151 indexer keys), stacks them on every step and hands the gathered
rows to the backend (`compressed_attention`, gpu/backend.py:233-254).  Here
the caches of `batch` requests stay in HBM ([batch][capacity][dim] each,
with per-request lengths on the device) and one decode step is one replayed
CUDA graph: the step's inputs are copied in from pinned memory, the new
rows are appended at each request's length (glmvx_dsa_append), the indexer
scores, stable top-k and absorbed MLA run on the device
(glmvx_dsa_decode_wait), and the attended latents and selections are copied
back.  The attention queries (most of the inbound bytes) travel on a second
stream while the append, indexer and top-k run; the attention stage waits
for them.

Semantics per request (model.py:136-176 `_index`, :205-221 the fused
attention branch): scores over all cached positions including the new one,
top-min(topk, length) positions with ties to the lower position, then
softmax(scale * (q_latent . latent + q_rope . rope_key)) over those rows
applied to the latents.
"""
import numpy as np

from . import runtime as rt


class DSADecoder:
    """Caches and one-step decode for `batch` requests of up to `capacity`
    positions.  Defaults are the GLM-DSA shapes: 64 heads, latent rank 512,
    rope 64, indexer 32 heads x 128, top-2048; scale (nope + rope)^-1/2 with
    nope 192 and index_scale index_dim^-1/2."""

    def __init__(self, backend, batch, capacity, *, heads=64, rank=512, rope_dim=64, index_heads=32, index_dim=128,
                 topk=2048, scale=None, index_scale=None):
        self.backend, self.lib = backend, backend.lib
        self.batch, self.capacity, self.heads, self.rank = int(batch), int(capacity), int(heads), int(rank)
        self.rope_dim, self.index_heads, self.index_dim, self.topk = (int(rope_dim), int(index_heads),
                                                                     int(index_dim), int(topk))
        self.scale = float(np.float32((192 + self.rope_dim) ** -0.5 if scale is None else scale))
        self.index_scale = float(np.float32(self.index_dim ** -0.5 if index_scale is None else index_scale))
        if min(self.batch, self.capacity, self.heads, self.index_heads, self.index_dim, self.topk) < 1:
            raise ValueError('DSA batch, capacity, heads, indexer shape and topk must be positive')
        if not 1 <= self.rank <= 512 or not 0 <= self.rope_dim <= 128 or self.topk > 4096:
            raise ValueError('DSA decode supports rank <= 512, rope_dim <= 128 and topk <= 4096')
        if not (np.isfinite(self.scale) and self.scale > 0 and np.isfinite(self.index_scale)):
            raise ValueError('DSA scales must be finite, the attention scale positive')
        backend._begin()
        B, T = self.batch, self.capacity
        self._bufs = []

        def dev(nbytes):
            buf = rt.DeviceBuffer(max(int(nbytes), 16))
            self._bufs.append(buf)
            return buf

        self.latents = dev(4 * B * T * self.rank)
        self.rope_keys = dev(4 * B * T * self.rope_dim)
        self.index_keys = dev(4 * B * T * self.index_dim)
        self.lens_dev = dev(4 * B)
        self.lens = np.zeros(B, np.int64)  # host mirror of the device lengths
        need = int(self.lib.glmvx_dsa_scratch_bytes(B, self.heads, self.rank, T, self.topk))
        if need < 0:
            raise ValueError('DSA scratch size')
        self._scratch, self._scratch_bytes = dev(need), need
        # I/O: the attention queries (copied on a second stream while the
        # append, indexer and top-k run), the append and indexer inputs and
        # the overflow flag (sent as 0 and read back), then the outputs
        # (attended latents, selections).
        H, R, P, IH, ID = self.heads, self.rank, self.rope_dim, self.index_heads, self.index_dim
        shapes = [('q_latent', np.float32, (B, H, R)), ('q_rope', np.float32, (B, H, P)),
                  ('new_latent', np.float32, (B, R)), ('new_rope', np.float32, (B, P)),
                  ('new_index_key', np.float32, (B, ID)), ('q_index', np.float32, (B, IH, ID)),
                  ('head_weights', np.float32, (B, IH)), ('full', np.int32, (1,)),
                  ('out', np.float32, (B, H, R)), ('selected', np.int32, (B, self.topk))]
        self._offs, off = {}, 0
        for name, dt, shape in shapes:
            self._offs[name] = (off, dt, shape)
            off += (4 * int(np.prod(shape)) + 255) & ~255
        self._io_bytes = off
        self._side, self._fork, self._queries_in = rt.Stream(), rt.Event(), rt.Event()
        self._longest = 0  # max(self.lens)
        self._host, self._dev = rt.HostBuffer(off), dev(off)
        self._io = {}
        for name, (o, dt, shape) in self._offs.items():
            n = int(np.prod(shape))
            self._io[name] = self._host.view(dt, o // 4 + n)[o // 4:].reshape(shape)
        self._io['full'][0] = 0
        self._upload(self.lens_dev, self.lens.astype(np.int32))
        self._graph = None

    def _ptr(self, name):
        return self._dev.ptr + self._offs[name][0]

    def _upload(self, buf, array, offset=0):
        buf.upload(np.ascontiguousarray(array), self.backend.stream.handle, offset)
        self.backend.stream.synchronize()

    def load(self, b, latents, rope_keys, index_keys):
        """Replace request b's cache with `count` prefilled rows
        (latents [count, rank], rope keys [count, rope_dim], index keys
        [count, index_dim])."""
        if not 0 <= b < self.batch:
            raise ValueError('request index out of range')
        lat = np.ascontiguousarray(latents, np.float32)
        rk = np.ascontiguousarray(rope_keys, np.float32).reshape(lat.shape[0], self.rope_dim)
        ik = np.ascontiguousarray(index_keys, np.float32)
        n = lat.shape[0]
        if lat.shape != (n, self.rank) or ik.shape != (n, self.index_dim):
            raise ValueError('cache rows must be [count, rank], [count, rope_dim] and [count, index_dim]')
        if n > self.capacity:
            raise ValueError('cache rows exceed capacity')
        row = b * self.capacity
        if n:
            self._upload(self.latents, lat, 4 * row * self.rank)
            if self.rope_dim:
                self._upload(self.rope_keys, rk, 4 * row * self.rope_dim)
            self._upload(self.index_keys, ik, 4 * row * self.index_dim)
        self.lens[b] = n
        self._longest = int(self.lens.max())
        self._upload(self.lens_dev, self.lens.astype(np.int32))

    def pinned_io(self):
        """Pinned views {'new_latent', 'new_rope', 'new_index_key', 'q_latent',
        'q_rope', 'q_index', 'head_weights'} to fill before step_pinned(), and
        {'out', 'selected'} holding its results until the next step."""
        return {k: v for k, v in self._io.items() if k != 'full'}

    def _step_graph(self):
        """The step as one graph: the append and indexer inputs (and a zero
        overflow flag) copied in on the stream; the attention queries copied
        in on a second stream, joined just before the attention stage; the
        flag and outputs copied back."""
        if self._graph is not None:
            return self._graph
        s = self.backend.stream.handle
        lib, B, T = self.lib, self.batch, self.capacity
        front, back = self._offs['new_latent'][0], self._offs['full'][0]
        g = rt.Graph(self.backend.stream)
        g.begin()
        try:
            rt.call('glmvx_memcpy_htod', self._dev.ptr + front, self._host.ptr + front,
                    self._offs['out'][0] - front, s)
            self._fork.record(s)
            self._side.wait_event(self._fork)
            rt.call('glmvx_memcpy_htod', self._dev.ptr, self._host.ptr, front, self._side.handle)
            self._queries_in.record(self._side)
            rt.check(lib, lib.glmvx_dsa_append(self.latents.ptr, self.rope_keys.ptr, self.index_keys.ptr,
                                               self.lens_dev.ptr, self._ptr('new_latent'), self._ptr('new_rope'),
                                               self._ptr('new_index_key'), B, T, self.rank, self.rope_dim,
                                               self.index_dim, self._ptr('full'), s), 'glmvx_dsa_append')
            rt.check(lib, lib.glmvx_dsa_decode_wait(
                self._ptr('out'), self._ptr('selected'), self._ptr('q_latent'), self._ptr('q_rope'),
                self._ptr('q_index'), self._ptr('head_weights'), self.latents.ptr, self.rope_keys.ptr,
                self.index_keys.ptr, self.lens_dev.ptr, B, self.heads, self.rank, self.rope_dim, self.index_heads,
                self.index_dim, T, self.topk, self.index_scale, self.scale, self._scratch.ptr, self._scratch_bytes,
                self._queries_in.handle, s), 'glmvx_dsa_decode_wait')
            rt.call('glmvx_memcpy_dtoh', self._host.ptr + back, self._dev.ptr + back, self._io_bytes - back, s)
        finally:
            g.end()
        self._graph = g
        return g

    def step_pinned(self):
        """One decode step for every request on the rows and queries already in
        pinned_io(): append, index, select, attend.  Returns the views
        (out [batch, heads, rank], selected [batch, topk], -1 padded)."""
        if self._longest >= self.capacity:
            raise ValueError('a request cache is full')
        self.backend._begin()
        full = self._io['full']
        full[0] = 0
        self._step_graph().launch()
        self.backend.stream.synchronize()
        if full[0]:
            raise RuntimeError('DSA cache overflow on the device')
        self.lens += 1
        self._longest += 1
        return self._io['out'], self._io['selected']

    def step(self, new_latent, new_rope, new_index_key, q_latent, q_rope, q_index, head_weights):
        """Copies the inputs ([batch, ...] as in pinned_io) into the pinned
        buffers, runs step_pinned() and returns copies of (out, selected)."""
        io = self._io
        for name, value in (('new_latent', new_latent), ('new_rope', new_rope), ('new_index_key', new_index_key),
                            ('q_latent', q_latent), ('q_rope', q_rope), ('q_index', q_index),
                            ('head_weights', head_weights)):
            value = np.asarray(value, np.float32)
            if value.size != io[name].size:
                raise ValueError(f'{name} must have shape {io[name].shape}')
            np.copyto(io[name], value.reshape(io[name].shape))
        out, sel = self.step_pinned()
        return out.copy(), sel.copy()

    def close(self):
        self.backend.stream.synchronize()
        if self._graph is not None:
            self._graph.close()
            self._graph = None
        self._host.close()
        for h in (self._side, self._fork, self._queries_in):
            h.close()
        for buf in self._bufs:
            buf.close()
        self._bufs = []
