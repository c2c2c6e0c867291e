"""Resident routed + shared MoE feed-forward layer on one B200.

Holds one sparse layer's weights in HBM -- the F32 router
(`mlp.gate.weight`) and its correction bias, packed GGML expert arrays
[experts][inter][hidden] (gate, up) and [experts][hidden][inter] (down), and
the shared expert -- and runs glmvx_moe_ffn: router, top-k, grouping by
expert, gate/up, SwiGLU fused into down, and the ascending-expert-id combine
with the shared expert added last.  Semantics are the reference model's
sparse feed-forward (glm_vx/model.py:289-324; grouped prefill form
glm_vx/prefill.py:44-81) for `tokens` independent rows.
"""
import ctypes as C

import numpy as np

from . import runtime as rt
from kernels.packed import LAYOUTS


def _u8(a):
    a = np.ascontiguousarray(a)
    return a.reshape(-1).view(np.uint8)


class MoELayer:
    def __init__(self, backend, router_w, router_bias, kind, gate, up, down, hidden, inter, top_k, scale,
                 shared=None):
        self.backend, self.kind = backend, int(kind)
        self.hidden, self.inter, self.top_k, self.scale = int(hidden), int(inter), int(top_k), float(scale)
        router_w = np.ascontiguousarray(router_w, dtype=np.float32)
        self.experts = router_w.shape[0]
        if router_w.shape != (self.experts, self.hidden) or np.shape(router_bias) != (self.experts,):
            raise ValueError('router weight must be [experts, hidden] and bias [experts]')
        block, size, _ = LAYOUTS[self.kind]
        if self.hidden % block or self.inter % block:
            raise ValueError('hidden and intermediate sizes must be block-aligned')
        gu = self.experts * self.inter * (self.hidden // block) * size
        dn = self.experts * self.hidden * (self.inter // block) * size
        for name, arr, n in (('gate', gate, gu), ('up', up, gu), ('down', down, dn)):
            if _u8(arr).nbytes != n:
                raise ValueError(f'{name} expert bytes do not match [experts, rows, cols] of format {self.kind}')
        backend._begin()
        s = backend.stream.handle
        self._buffers = []

        def upload(arr):
            arr = np.ascontiguousarray(arr)
            buf = rt.DeviceBuffer(max(arr.nbytes, 16))
            buf.upload(arr, s)
            self._buffers.append(buf)
            return buf.ptr

        self.router_w = upload(router_w)
        self.router_bias = upload(np.asarray(router_bias, np.float32))
        self.gate, self.up, self.down = upload(_u8(gate)), upload(_u8(up)), upload(_u8(down))
        if shared is not None:
            sg, su, sd = shared
            one_gu = self.inter * (self.hidden // block) * size
            one_dn = self.hidden * (self.inter // block) * size
            if _u8(sg).nbytes != one_gu or _u8(su).nbytes != one_gu or _u8(sd).nbytes != one_dn:
                raise ValueError('shared expert bytes do not match one expert')
            self.shared = (upload(_u8(sg)), upload(_u8(su)), upload(_u8(sd)))
        else:
            self.shared = (None, None, None)
        backend.stream.synchronize()
        self._ws, self._ws_bytes, self._io = None, 0, None

    def workspace_bytes(self, tokens):
        cache = self.__dict__.setdefault('_ws_need', {})
        if tokens not in cache:
            cache[tokens] = int(self.backend.lib.glmvx_moe_workspace_bytes(
                tokens, self.hidden, self.inter, self.experts, self.top_k, int(self.shared[0] is not None)))
        return cache[tokens]

    def _workspace(self, tokens):
        need = self.workspace_bytes(tokens)
        if need > self._ws_bytes:
            if self._ws is not None:
                self.backend.stream.synchronize()
                self._drop_graphs()
                self._ws.close()
            self._ws, self._ws_bytes = rt.DeviceBuffer(need), need
        return self._ws.ptr

    def _drop_graphs(self):
        for g in self.__dict__.get('_graphs', {}).values():
            g.close()
        self._graphs = {}

    _IO_SLOTS = ('x', 'flag', 'y', 'ids', 'weights', 'err')

    def _io_layout(self, tokens):
        """Byte offsets {'x', 'flag', 'y', 'ids', 'weights', 'err'} in the
        layer's I/O buffers (pinned host + device, 256-byte aligned), grown on
        demand.  The non-finite-output flag sits between the input rows and
        the outputs: the step's one host-to-device copy (x and a zero flag)
        clears it and its first device-to-host copy (flag to weights) returns
        it."""
        n, k = 4 * tokens * self.hidden, 4 * tokens * self.top_k
        offs, off = {}, 0
        for name, size in zip(self._IO_SLOTS, (n, 4, n, k, k, 4)):
            offs[name] = off
            off += (size + 255) & ~255
        if off > self.__dict__.get('_io_cap', 0):
            self.backend.stream.synchronize()
            self._drop_graphs()
            for buf in self.__dict__.get('_io_bufs', ()):
                buf.close()
            self._io_bufs = (rt.HostBuffer(off), rt.DeviceBuffer(off))
            self._io_cap = off
            self._io_views = {}
        return offs

    def step_copy_bytes(self, tokens):
        """(host-to-device, device-to-host) bytes that one forward_pinned(tokens)
        step copies: the rows and the flag in; the flag, outputs and routing,
        then the device error word, out."""
        o = self._io_layout(tokens)
        return o['flag'] + 4 - o['x'], o['weights'] + 4 * tokens * self.top_k - o['flag'] + 4

    def pinned_io(self, tokens):
        """Pinned host views for a `tokens`-row step: {'x', 'y', 'ids',
        'weights'}.  Write the rows into 'x' and call forward_pinned(tokens);
        the other views then hold its results until the next call."""
        return self._pinned(tokens)[0]

    def _pinned(self, tokens):
        """(pinned_io views, flag word, error word) of a `tokens`-row step,
        made once per buffer layout."""
        offs = self._io_layout(tokens)
        cached = self._io_views.get(tokens)
        if cached is None:
            host = self._io_bufs[0]
            n, k = tokens * self.hidden, tokens * self.top_k

            def view(name, dtype, count, shape):
                o = offs[name] // 4
                return host.view(dtype, o + count)[o:].reshape(shape)

            views = {'x': view('x', np.float32, n, (tokens, self.hidden)),
                     'y': view('y', np.float32, n, (tokens, self.hidden)),
                     'ids': view('ids', np.int32, k, (tokens, self.top_k)),
                     'weights': view('weights', np.float32, k, (tokens, self.top_k))}
            cached = (views, C.c_uint32.from_address(host.ptr + offs['flag']),
                      C.c_int32.from_address(host.ptr + offs['err']))
            self._io_views[tokens] = cached
        return cached

    def _step_graph(self, tokens):
        """CUDA graph of one step on the I/O buffers: copy the token rows (and
        a zero flag) in, the layer's launches, flag a non-finite output, copy
        the flag, outputs and routing back, then the device error word.
        Replayed per call so the GPU runs the step without host gaps;
        captured again when the buffers or the workspace move."""
        b = self.backend
        offs = self._io_layout(tokens)
        self._workspace(tokens)  # allocated before capture
        host, dev = self._io_bufs
        key = (tokens, host.ptr, dev.ptr, self._ws.ptr)
        graphs = self.__dict__.setdefault('_graphs', {})
        if key in graphs:
            return graphs[key]
        if any(k[1:] != key[1:] for k in graphs):
            self._drop_graphs()
            graphs = self._graphs
        s = b.stream.handle
        h2d, d2h = self.step_copy_bytes(tokens)
        g = rt.Graph(b.stream)
        g.begin()
        try:
            rt.call('glmvx_memcpy_htod', dev.ptr + offs['x'], host.ptr + offs['x'], h2d, s)
            self.forward_device(dev.ptr + offs['y'], dev.ptr + offs['x'], tokens, dev.ptr + offs['ids'],
                                dev.ptr + offs['weights'])
            rt.call('glmvx_nonfinite_flag', dev.ptr + offs['y'], tokens * self.hidden, dev.ptr + offs['flag'], s)
            rt.call('glmvx_memcpy_dtoh', host.ptr + offs['flag'], dev.ptr + offs['flag'], d2h - 4, s)
            rt.call('glmvx_memcpy_dtoh', host.ptr + offs['err'], b.device.error_address(), 4, s)
        finally:
            g.end()
        graphs[key] = g
        return g

    def forward_device(self, y, x, tokens, ids=None, weights=None, stream=None):
        """Device pointers in and out; asynchronous on `stream` (default: the backend's)."""
        ws = self._workspace(tokens)
        rt.check(self.backend.lib, self.backend.lib.glmvx_moe_ffn(
            y, x, tokens, self.hidden, self.inter, self.router_w, self.router_bias, self.experts, self.top_k,
            self.scale, self.kind, self.gate, self.up, self.down, *self.shared, ws, self._ws_bytes, ids, weights,
            stream if stream is not None else self.backend.stream.handle), 'glmvx_moe_ffn')

    def forward_pinned(self, tokens):
        """One step on the rows already in pinned_io(tokens)['x'] -> views
        (y, ids, weights) of pinned_io(tokens), valid until the next call.
        Raises like forward() on non-finite inputs or outputs."""
        b = self.backend
        b._begin()
        io, flag, err = self._pinned(tokens)
        if tokens == 0:
            return io['y'], io['ids'], io['weights']
        g = self._step_graph(tokens)
        flag.value = 0  # copied in with the rows
        g.launch()
        b.stream.synchronize()
        if err.value:
            b.device.check_device_error()
        # Non-finite inputs run safely (the router ranks NaN scores last) and
        # give non-finite outputs, so one check after the step covers both;
        # a kernel after the layer flags a non-finite output on the device.
        if flag.value:
            if not np.isfinite(io['x']).all():
                raise ValueError('MoE input must be finite')
            raise ValueError('nonfinite MoE output')
        return io['y'], io['ids'], io['weights']

    def forward(self, x):
        """x [tokens, hidden] f32 -> (y [tokens, hidden], ids [tokens, k], weights [tokens, k])."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        if x.ndim != 2 or x.shape[1] != self.hidden:
            raise ValueError('MoE input must be [tokens, hidden]')
        T = x.shape[0]
        if T == 0:
            return (np.empty_like(x), np.empty((0, self.top_k), np.int32), np.empty((0, self.top_k), np.float32))
        self.backend._begin()
        np.copyto(self.pinned_io(T)['x'], x)
        y, ids, wts = self.forward_pinned(T)
        return y.copy(), ids.copy(), wts.copy()

    def close(self):
        self.backend.stream.synchronize()
        self._drop_graphs()
        for buf in self.__dict__.pop('_io_bufs', ()):
            buf.close()
        self._io_cap, self._io_views = 0, {}
        for buf in self._buffers + ([self._ws] if self._ws is not None else []):
            buf.close()
        self._buffers, self._ws = [], None
