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
                self._ws.close()
            self._ws, self._ws_bytes = rt.DeviceBuffer(need), need
        return self._ws.ptr

    def forward_device(self, y, x, tokens, ids=None, weights=None, stream=None):
        """Device pointers in and out; asynchronous on `stream` (default: the backend's)."""
        ws = self._workspace(tokens)
        rt.check(self.backend.lib, self.backend.lib.glmvx_moe_ffn(
            y, x, tokens, self.hidden, self.inter, self.router_w, self.router_bias, self.experts, self.top_k,
            self.scale, self.kind, self.gate, self.up, self.down, *self.shared, ws, self._ws_bytes, ids, weights,
            stream if stream is not None else self.backend.stream.handle), 'glmvx_moe_ffn')

    def forward(self, x):
        """x [tokens, hidden] f32 -> (y [tokens, hidden], ids [tokens, k], weights [tokens, k])."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        if x.ndim != 2 or x.shape[1] != self.hidden:
            raise ValueError('MoE input must be [tokens, hidden]')
        if not np.isfinite(x).all():
            raise ValueError('MoE input must be finite')
        b = self.backend
        b._begin()
        T = x.shape[0]
        y = np.empty_like(x)
        ids = np.empty((T, self.top_k), np.int32)
        wts = np.empty((T, self.top_k), np.float32)
        if T == 0:
            return y, ids, wts
        (xd,), (yd, idd, wd, _), offs = b._stage([x], [y.nbytes, ids.nbytes, wts.nbytes, 4])
        self.forward_device(yd, xd, T, idd, wd)
        b._fetch_checked(offs[:3], [y, ids, wts], offs[3])
        if not np.isfinite(y).all():
            raise ValueError('nonfinite MoE output')
        return y, ids, wts

    def close(self):
        self.backend.stream.synchronize()
        for buf in self._buffers + ([self._ws] if self._ws is not None else []):
            buf.close()
        self._buffers, self._ws = [], None
