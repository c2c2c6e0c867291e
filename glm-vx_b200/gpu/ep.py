"""Expert-parallel routed + shared MoE layer over peer memory (csrc/ep.cu).

The reference runs every expert of a sparse layer in one process
(glm_vx/model.py:289-324).  Here the routed experts are sharded over the
GPUs of one node -- expert e on rank e // (experts / world) -- while the F32
router and the shared expert are replicated, and a layer step runs entirely
on the device: route, store each (token, expert) pair's prepared row into
the owner's mailbox over NVLink, the owner's tensor-core expert jobs with
their down outputs stored straight back into the sender's mailbox, and the
ascending-expert-id combine.  No collective library, no PyTorch, no host
round trip inside a step; a step is one replayable CUDA graph per rank.

Setting up needs one exchange of 64-byte CUDA IPC handles between the rank
processes (`connect_ipc` with any all-gather of bytes: `FileBootstrap`
below, or a launcher's own store).  Ranks that share one process and one
device (tests on a single GPU) connect with plain pointers instead
(`emulated_ranks` / `emulated_forward`).
"""
import ctypes as C
import os
import time
from pathlib import Path

import numpy as np

from . import runtime as rt
from kernels.packed import LAYOUTS


def experts_per_rank(experts, world):
    if experts % world:
        raise ValueError(f'{experts} experts do not split evenly over {world} ranks')
    return experts // world


def _u8(a):
    return np.ascontiguousarray(a).reshape(-1).view(np.uint8)


class FileBootstrap:
    """All-gather of small byte strings between the rank processes of one
    host through a directory they share (no network, no torch): each call
    writes this rank's bytes to `<dir>/<tag>.<call>.<rank>` and waits (up to
    `timeout` seconds) for every rank's file of the same call."""

    def __init__(self, directory, rank, world, tag='ep', timeout=120.0):
        self.dir, self.rank, self.world, self.tag = Path(directory), int(rank), int(world), str(tag)
        self.timeout, self.calls = float(timeout), 0
        self.dir.mkdir(parents=True, exist_ok=True)

    def _path(self, call, rank):
        return self.dir / f'{self.tag}.{call}.{rank}'

    def allgather(self, data):
        call = self.calls
        self.calls += 1
        tmp = self.dir / f'.{self.tag}.{call}.{self.rank}.tmp'
        tmp.write_bytes(bytes(data))
        os.replace(tmp, self._path(call, self.rank))
        deadline = time.monotonic() + self.timeout
        out = [None] * self.world
        while True:
            for r in range(self.world):
                if out[r] is None and self._path(call, r).exists():
                    out[r] = self._path(call, r).read_bytes()
            if all(o is not None for o in out):
                return out
            if time.monotonic() > deadline:
                missing = [r for r in range(self.world) if out[r] is None]
                raise TimeoutError(f'bootstrap call {call}: ranks {missing} did not arrive in {self.timeout} s')
            time.sleep(0.01)

    def barrier(self):
        self.allgather(b'')


class ExpertParallelLayer:
    """This rank's part of a sparse layer: `gate`/`up`/`down` hold its
    experts [rank*E/world, (rank+1)*E/world) as packed GGML stacks
    ([experts/world][rows][row_bytes]); the router, its bias and the shared
    expert are the full, replicated arrays.  Steps of up to `max_tokens`
    token rows per rank (world * max_tokens * top_k <= 4096)."""

    def __init__(self, backend, rank, world, router_w, router_bias, kind, gate, up, down, experts, hidden, inter,
                 top_k, scale, shared=None, max_tokens=32, device_weights=False):
        """device_weights: router_w, router_bias, gate, up, down and shared
        are device addresses (ints) of resident arrays the caller keeps alive,
        laid out as the host arrays would be; nothing is uploaded."""
        self.backend, self.lib = backend, backend.lib
        self.rank, self.world = int(rank), int(world)
        self.kind, self.experts, self.hidden, self.inter = int(kind), int(experts), int(hidden), int(inter)
        self.top_k, self.scale, self.max_tokens = int(top_k), float(scale), int(max_tokens)
        self.per_rank = experts_per_rank(self.experts, self.world)
        self._buffers = []
        if device_weights:
            self.router_w, self.router_bias = int(router_w), int(router_bias)
            self.gate, self.up, self.down = int(gate), int(up), int(down)
            self.shared = tuple(int(p) for p in shared) if shared is not None else (None, None, None)
            self._create()
            return
        block, size, _ = LAYOUTS[self.kind]
        if self.hidden % block or self.inter % block:
            raise ValueError('hidden and intermediate sizes must be block-aligned')
        one_gu = self.inter * (self.hidden // block) * size
        one_dn = self.hidden * (self.inter // block) * size
        for name, arr, n in (('gate', gate, one_gu), ('up', up, one_gu), ('down', down, one_dn)):
            if _u8(arr).nbytes != self.per_rank * n:
                raise ValueError(f"{name} must hold this rank's {self.per_rank} experts of format {self.kind}")
        router_w = np.ascontiguousarray(router_w, dtype=np.float32)
        if router_w.shape != (self.experts, self.hidden) or np.shape(router_bias) != (self.experts,):
            raise ValueError('router weight must be [experts, hidden] and bias [experts]')
        backend._begin()
        s = backend.stream.handle

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
            sg, su, sd = (_u8(a) for a in shared)
            if sg.nbytes != one_gu or su.nbytes != one_gu or sd.nbytes != one_dn:
                raise ValueError('shared expert bytes do not match one expert')
            self.shared = (upload(sg), upload(su), upload(sd))
        else:
            self.shared = (None, None, None)
        backend.stream.synchronize()
        self._create()

    def _create(self):
        handle = C.c_void_p()
        rt.check(self.lib, self.lib.glmvx_ep_create(
            C.byref(handle), self.rank, self.world, self.max_tokens, self.hidden, self.inter, self.experts, self.top_k,
            self.scale, self.kind, self.router_w, self.router_bias, self.gate, self.up, self.down, *self.shared),
            'glmvx_ep_create')
        self.handle = handle.value
        self._mapped, self._graphs, self._io = [], {}, None

    # ------------------------------------------------------------- set-up
    def mailbox(self):
        base, nbytes = C.c_void_p(), C.c_uint64()
        rt.check(self.lib, self.lib.glmvx_ep_mailbox(self.handle, C.byref(base), C.byref(nbytes)), 'glmvx_ep_mailbox')
        return base.value, nbytes.value

    def connect(self, mailboxes):
        """Mailbox addresses of every rank in rank order, as this process
        sees them (own included)."""
        if len(mailboxes) != self.world:
            raise ValueError('one mailbox per rank')
        arr = (C.c_void_p * self.world)(*[int(m) for m in mailboxes])
        rt.check(self.lib, self.lib.glmvx_ep_connect(self.handle, arr), 'glmvx_ep_connect')

    def connect_ipc(self, allgather):
        """Swap CUDA IPC handles of the mailboxes with the other rank
        processes through `allgather(bytes) -> [bytes per rank]` and map
        theirs."""
        own, _ = self.mailbox()
        handle = (C.c_uint8 * 64)()
        rt.call('glmvx_ipc_handle', own, handle)
        handles = allgather(bytes(handle))
        bases = []
        for r, h in enumerate(handles):
            if r == self.rank:
                bases.append(own)
                continue
            p = C.c_void_p()
            rt.call('glmvx_ipc_open', (C.c_uint8 * 64).from_buffer_copy(h), C.byref(p))
            self._mapped.append(p.value)
            bases.append(p.value)
        self.connect(bases)

    # -------------------------------------------------------------- steps
    def _stream(self, stream):
        return stream if stream is not None else self.backend.stream.handle

    def dispatch(self, x, tokens, ids=None, weights=None, stream=None):
        rt.check(self.lib, self.lib.glmvx_ep_dispatch(self.handle, x, tokens, ids, weights, self._stream(stream)),
                 'glmvx_ep_dispatch')

    def run_experts(self, tokens, stream=None):
        rt.check(self.lib, self.lib.glmvx_ep_experts(self.handle, tokens, self._stream(stream)), 'glmvx_ep_experts')

    def combine(self, y, tokens, stream=None):
        rt.check(self.lib, self.lib.glmvx_ep_combine(self.handle, y, tokens, self._stream(stream)), 'glmvx_ep_combine')

    def forward_device(self, y, x, tokens, ids=None, weights=None, stream=None):
        """One step on device pointers (every rank must step together)."""
        rt.check(self.lib, self.lib.glmvx_ep_step(self.handle, y, x, tokens, ids, weights, self._stream(stream)),
                 'glmvx_ep_step')

    _IO = ('x', 'flag', 'y', 'ids', 'weights', 'err')

    def _io_layout(self, tokens):
        n, k = 4 * tokens * self.hidden, 4 * tokens * self.top_k
        offs, off = {}, 0
        for name, size in zip(self._IO, (n, 4, n, k, k, 4)):
            offs[name] = off
            off += (size + 255) & ~255
        if self._io is None or off > self._io[0].nbytes:
            self.backend.stream.synchronize()
            self._drop_graphs()
            if self._io is not None:
                for b in self._io:
                    b.close()
            self._io = (rt.HostBuffer(off), rt.DeviceBuffer(off))
            self._views = {}
        return offs

    def step_copy_bytes(self, tokens):
        """(host-to-device, device-to-host) bytes of one forward_pinned step."""
        o = self._io_layout(tokens)
        return o['flag'] + 4 - o['x'], o['weights'] + 4 * tokens * self.top_k - o['flag'] + 4

    def pinned_io(self, tokens):
        """Pinned host views {'x', 'y', 'ids', 'weights'} of a `tokens`-row step."""
        return self._pinned(tokens)[0]

    def _pinned(self, tokens):
        offs = self._io_layout(tokens)
        if tokens not in self._views:
            host = self._io[0]

            def view(name, dtype, count, shape):
                o = offs[name] // 4
                return host.view(dtype, o + count)[o:].reshape(shape)

            n, k = tokens * self.hidden, tokens * self.top_k
            self._views[tokens] = ({'x': view('x', np.float32, n, (tokens, self.hidden)),
                                    'y': view('y', np.float32, n, (tokens, self.hidden)),
                                    'ids': view('ids', np.int32, k, (tokens, self.top_k)),
                                    'weights': view('weights', np.float32, k, (tokens, self.top_k))},
                                   C.c_uint32.from_address(host.ptr + offs['flag']),
                                   C.c_int32.from_address(host.ptr + offs['err']))
        return self._views[tokens]

    def _drop_graphs(self):
        for g in self._graphs.values():
            g.close()
        self._graphs = {}

    def _step_graph(self, tokens):
        """Graph of one step on the pinned I/O buffers: rows (and a zero
        non-finite flag) in, the step, the flag kernel, flag + outputs +
        routing out, then the device error word."""
        offs = self._io_layout(tokens)
        host, dev = self._io
        key = (tokens, host.ptr, dev.ptr)
        if key not in self._graphs:
            s = self.backend.stream.handle
            h2d, d2h = self.step_copy_bytes(tokens)
            g = rt.Graph(self.backend.stream)
            g.begin()
            try:
                rt.call('glmvx_memcpy_htod', dev.ptr + offs['x'], host.ptr + offs['x'], h2d, s)
                self.forward_device(dev.ptr + offs['y'], dev.ptr + offs['x'], tokens, dev.ptr + offs['ids'],
                                    dev.ptr + offs['weights'])
                rt.call('glmvx_nonfinite_flag', dev.ptr + offs['y'], tokens * self.hidden, dev.ptr + offs['flag'], s)
                rt.call('glmvx_memcpy_dtoh', host.ptr + offs['flag'], dev.ptr + offs['flag'], d2h - 4, s)
                rt.call('glmvx_memcpy_dtoh', host.ptr + offs['err'], self.backend.device.error_address(), 4, s)
            finally:
                g.end()
            self._graphs[key] = g
        return self._graphs[key]

    def forward_pinned(self, tokens):
        """One step on the rows in pinned_io(tokens)['x'] -> views (y, ids,
        weights), valid until the next call.  Every rank calls it for the
        same step; raises on a device error (a peer that did not arrive
        within 2 s) or a non-finite output."""
        b = self.backend
        b._begin()
        if not 0 <= tokens <= self.max_tokens:
            raise ValueError(f'tokens must be 0..{self.max_tokens}')
        io, flag, err = self._pinned(max(tokens, 1))
        if tokens == 0:
            self.forward_device(None, None, 0)
            b.stream.synchronize()
            b.device.check_device_error()
            return io['y'][:0], io['ids'][:0], io['weights'][:0]
        g = self._step_graph(tokens)
        flag.value = 0
        g.launch()
        b.stream.synchronize()
        if err.value:
            b.device.check_device_error()
        if flag.value:
            if not np.isfinite(io['x']).all():
                raise ValueError('MoE input must be finite')
            raise ValueError('nonfinite MoE output')
        return io['y'], io['ids'], io['weights']

    def forward(self, x):
        """x [tokens, hidden] f32 (host) -> (y, ids, weights) host copies."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        if x.ndim != 2 or x.shape[1] != self.hidden:
            raise ValueError('MoE input must be [tokens, hidden]')
        T = x.shape[0]
        if T:
            np.copyto(self.pinned_io(T)['x'], x)
        y, ids, w = self.forward_pinned(T)
        return y.copy(), ids.copy(), w.copy()

    def close(self, barrier=None):
        """Unmap the peers' mailboxes, wait at `barrier` (every rank has
        unmapped this one) and free this rank's layer."""
        if getattr(self, 'handle', None) is None:
            return
        self.backend.stream.synchronize()
        self._drop_graphs()
        for p in self._mapped:
            rt.call('glmvx_ipc_close', p)
        self._mapped = []
        if barrier is not None:
            barrier()
        rt.call('glmvx_ep_destroy', self.handle)
        self.handle = None
        if self._io is not None:
            for b in self._io:
                b.close()
            self._io = None
        for b in self._buffers:
            b.close()
        self._buffers = []


def split_layer(layer, world, rank):
    """This rank's expert stacks of a full layer's host arrays (dict with
    'gate', 'up', 'down' [experts][...] bytes and 'router')."""
    experts = np.shape(layer['router'])[0]
    per = experts_per_rank(experts, world)

    def part(a):
        a = _u8(a)
        one = a.nbytes // experts
        return a[rank * per * one:(rank + 1) * per * one]

    return part(layer['gate']), part(layer['up']), part(layer['down'])


def emulated_ranks(backend, world, layer, kind, hidden, inter, top_k, scale, max_tokens):
    """`world` ranks of one layer in THIS process on one device, connected
    by plain device pointers (a single-GPU stand-in for world GPUs, for
    testing the multi-rank data layout).  Step them with emulated_forward."""
    ranks = []
    for r in range(world):
        g, u, d = split_layer(layer, world, r)
        ranks.append(ExpertParallelLayer(backend, r, world, layer['router'], layer['bias'], kind, g, u, d,
                                         np.shape(layer['router'])[0], hidden, inter, top_k, scale,
                                         shared=layer.get('shared'), max_tokens=max_tokens))
    boxes = [r.mailbox()[0] for r in ranks]
    for r in ranks:
        r.connect(boxes)
    return ranks


def emulated_forward(ranks, xs):
    """One step of emulated ranks: xs[r] [T_r, hidden] host rows of rank r ->
    [(y, ids, weights)] per rank.  The three phases are issued rank by rank
    on one stream -- every dispatch, then every rank's experts, then every
    combine -- so each device-side wait is already satisfied when it runs
    (kernels that wait on each other never run concurrently here)."""
    b = ranks[0].backend
    s = b.stream.handle
    bufs = []
    try:
        for lay, x in zip(ranks, xs):
            x = np.ascontiguousarray(x, np.float32)
            T = x.shape[0]
            xd, yd = rt.DeviceBuffer(max(x.nbytes, 16)), rt.DeviceBuffer(max(x.nbytes, 16))
            idd, wd = rt.DeviceBuffer(max(4 * T * lay.top_k, 16)), rt.DeviceBuffer(max(4 * T * lay.top_k, 16))
            if T:
                xd.upload(x, s)
            bufs.append((T, xd, yd, idd, wd))
        for lay, (T, xd, _, idd, wd) in zip(ranks, bufs):
            lay.dispatch(xd.ptr, T, idd.ptr, wd.ptr)
        for lay, (T, *_) in zip(ranks, bufs):
            lay.run_experts(T)
        for lay, (T, _, yd, _, _) in zip(ranks, bufs):
            lay.combine(yd.ptr, T)
        b.stream.synchronize()
        b.device.check_device_error()
        out = []
        for lay, (T, _, yd, idd, wd) in zip(ranks, bufs):
            y = np.empty((T, lay.hidden), np.float32)
            ids = np.empty((T, lay.top_k), np.int32)
            w = np.empty((T, lay.top_k), np.float32)
            if T:
                yd.download(y)
                idd.download(ids)
                wd.download(w)
            out.append((y, ids, w))
        return out
    finally:
        for _, *bs in bufs:
            for buf in bs:
                buf.close()
