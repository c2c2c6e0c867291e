"""Expert parallelism for the routed + shared MoE layer.

The reference runs every expert of a layer in one process
(glm_vx/model.py:289-324).  Here the routed experts are sharded over the
ranks of a process group -- expert e lives on rank e // (experts / world) --
while the router and the shared expert are replicated.  One layer step for
the T token rows a rank owns:

  1. route locally (F32 router logits, sigmoid top-k with bias);
  2. plan: every (token, slot) pair goes to the rank that owns its expert;
     pairs are sent grouped by destination, in (token, slot) order;
  3. exchange the pair counts, then the token rows and their expert ids
     (all_to_all_single over the group: NCCL between GPUs, gloo on CPU);
  4. the owner runs its experts on the received rows (grouped by expert);
  5. a reverse all_to_all_single returns one output row per pair;
  6. the routing rank sums each token's pair outputs in ascending expert id,
     weighted, and adds the shared expert's output last -- the reference's
     order, so the result does not depend on the number of ranks.

The planning and the exchange are host logic written once; the compute is
supplied by the caller (`ExpertParallelMoE` uses the CUDA library; the CPU
tests plug in the oracle).
"""

import ctypes as C

import numpy as np

try:  # plumbing only: collectives and device tensors for the exchange buffers
    import torch
    import torch.distributed as dist
except ImportError:  # pragma: no cover - the exchange needs torch.distributed
    torch = dist = None


def experts_per_rank(experts, world):
    if experts % world:
        raise ValueError(f'{experts} experts do not split evenly over {world} ranks')
    return experts // world


def dispatch_plan(ids, per_rank, world):
    """ids int [T, k] global expert ids -> (order, counts): `order` lists the
    flattened pair indices t*k+j grouped by destination rank (stable, so in
    (token, slot) order within a rank); counts[d] pairs go to rank d."""
    ids = np.asarray(ids)
    dest = (ids.reshape(-1) // per_rank).astype(np.int64)
    if dest.size and (dest.min() < 0 or dest.max() >= world):
        raise ValueError('expert id outside the sharded range')
    order = np.argsort(dest, kind='stable')
    return order, np.bincount(dest, minlength=world).astype(np.int64)


def combine_plan(ids, wts, order):
    """Per token, the positions (in the send order) of its pair outputs and
    their weights, in ascending expert id (glm_vx/model.py:305-316)."""
    ids, wts = np.asarray(ids), np.asarray(wts, np.float32)
    T, k = ids.shape
    pos = np.empty(T * k, np.int64)
    pos[order] = np.arange(T * k)
    srt = np.argsort(ids, axis=1, kind='stable')
    rows = np.arange(T)[:, None]
    return pos.reshape(T, k)[rows, srt].astype(np.int32), wts[rows, srt].astype(np.float32)


class Exchange:
    """all_to_all_single over a process group for tensors on `device`."""

    def __init__(self, group=None, device='cpu'):
        self.group, self.device = group, device
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)

    def counts(self, send_counts):
        send = torch.as_tensor(np.asarray(send_counts, np.int64), device=self.device)
        recv = torch.empty_like(send)
        dist.all_to_all_single(recv, send, group=self.group)
        return recv.cpu().numpy()

    def rows(self, send, send_counts, recv_counts):
        recv = send.new_empty((int(np.sum(recv_counts)),) + tuple(send.shape[1:]))
        dist.all_to_all_single(recv, send.contiguous(), [int(c) for c in recv_counts],
                               [int(c) for c in send_counts], group=self.group)
        return recv


def peer_layout(M, send_counts, rank):
    """Where this rank's rows land in a peer exchange, given the count matrix
    M[s, d] (rows rank s sends to rank d in the forward direction):
    (S, dst_rows, total) with S the matrix of this exchange (M forward, M.T
    when the rows go back), dst_rows[d] the row of rank d's mailbox at which
    this rank's rows start (the senders before it, in rank order -- the
    concatenation order of all_to_all_single), total the rows this rank
    receives."""
    M = np.asarray(M, np.int64)
    send_counts = np.asarray(send_counts, np.int64)
    if np.array_equal(send_counts, M[rank]):
        S = M
    elif np.array_equal(send_counts, M[:, rank]):
        S = M.T
    else:
        raise ValueError('rows() counts match neither direction of the last counts()')
    dst_rows = [int(S[:rank, d].sum()) for d in range(S.shape[0])]
    return S, dst_rows, int(S[:, rank].sum())


class _DeviceView:
    """Zero-copy torch view of raw device memory (__cuda_array_interface__)."""

    def __init__(self, ptr, nbytes):
        self.__cuda_array_interface__ = {'shape': (int(nbytes),), 'typestr': '|u1', 'data': (int(ptr), False),
                                         'version': 3, 'strides': None}


def _pad16(n):
    return (int(n) + 15) // 16 * 16


class PeerExchange:
    """The interface of Exchange over peer memory instead of a collective
    library (csrc/p2p.cu): every rank cudaMallocs a mailbox, the ranks swap
    64-byte CUDA IPC handles once and map each other's mailboxes, and each
    exchange is three launches on the current stream -- a scatter kernel
    storing this rank's rows straight into the destinations' mailboxes over
    NVLink, a signal kernel publishing the step's epoch in each destination's
    flag slot for this rank (release, system scope), and a wait kernel
    (acquire, bounded to 2 s) until every sender's flag reached the epoch.

    counts() shares the whole send-count matrix (a row per rank, in every
    mailbox) and returns it to the host, as all_to_all of the counts does;
    rows() then knows every rank's offsets (peer_layout): forward rows land
    in each destination in sender order, rows sent back (send counts = the
    received counts) in each sender's order of destinations.  The rows
    returned are a view of this rank's mailbox, valid until the next step's
    counts() (every rank finishes a step before any rank's next counts()
    completes).  Up to three rows() calls per counts(); at most `max_rows`
    rows received per call, `row_bytes` bytes each (narrower rows are padded
    to 16 bytes).  Plain peer stores: no multicast object."""

    REGIONS = 3

    def __init__(self, group, device, max_rows, row_bytes):
        from . import runtime as rt
        self.rt, self.lib, self.group, self.device = rt, rt.library(), group, device
        self.world, self.rank = dist.get_world_size(group), dist.get_rank(group)
        if self.world > 8:
            raise ValueError('peer exchange supports up to 8 ranks')
        rt.call('glmvx_set_device', device.index)
        self.max_rows, self.row_cap = int(max_rows), _pad16(row_bytes)
        W = self.world
        self.count_row = _pad16(8 * W)
        self.flags_off = (W * self.count_row + 255) // 256 * 256
        self.data_off = (self.flags_off + (self.REGIONS + 1) * W * 4 + 255) // 256 * 256
        self.region_bytes = (self.max_rows * self.row_cap + 255) // 256 * 256
        total = self.data_off + self.REGIONS * self.region_bytes
        self.mail = rt.DeviceBuffer(total)
        rt.call('glmvx_memset', self.mail.ptr, 0, self.data_off, None)
        rt.call('glmvx_device_synchronize')
        handle = (C.c_uint8 * 64)()
        rt.call('glmvx_ipc_handle', self.mail.ptr, handle)
        handles = [None] * W
        dist.all_gather_object(handles, bytes(handle), group=group)
        self.base = []
        for d in range(W):
            if d == self.rank:
                self.base.append(self.mail.ptr)
            else:
                p = C.c_void_p()
                rt.call('glmvx_ipc_open', (C.c_uint8 * 64).from_buffer_copy(handles[d]), C.byref(p))
                self.base.append(p.value)
        self.view = torch.as_tensor(_DeviceView(self.mail.ptr, total), device=device)
        self.stage = rt.DeviceBuffer(W * self.count_row)
        self.epoch, self.call, self.M = 0, 0, None
        dist.barrier(group)  # every mailbox zeroed and mapped before any store

    def _stream(self):
        return torch.cuda.current_stream(self.device).cuda_stream

    def _ptrs(self, vals):
        return (C.c_void_p * self.world)(*[int(v) for v in vals])

    def _i64(self, vals):
        return (C.c_int64 * self.world)(*[int(v) for v in vals])

    def _exchange_done(self, region):
        """Signal this rank's stores of `region` to every peer, then wait for
        every sender's stores into this rank's mailbox."""
        W, s = self.world, self._stream()
        slots = [self.base[d] + self.flags_off + (region * W + self.rank) * 4 for d in range(W)]
        self.rt.call('glmvx_p2p_signal', self._ptrs(slots), W, self.epoch, s)
        self.rt.call('glmvx_p2p_wait', self.mail.ptr + self.flags_off + region * W * 4, W, self.epoch, s)

    def counts(self, send_counts):
        W, s = self.world, self._stream()
        self.epoch = (self.epoch + 1) & 0xFFFFFFFF
        self.call = 0
        row = np.zeros(self.count_row // 8, np.int64)
        row[:W] = np.asarray(send_counts, np.int64)
        stage = np.ascontiguousarray(np.tile(row, (W, 1)))  # one copy of the row per destination
        self.rt.call('glmvx_memcpy_htod', self.stage.ptr, stage.ctypes.data, stage.nbytes, s)
        dst = [self.base[d] + self.rank * self.count_row for d in range(W)]
        self.rt.call('glmvx_p2p_scatter', self.stage.ptr, self.count_row, self._ptrs(dst), self._i64([1] * W), None,
                     W, s)
        self._exchange_done(0)
        m = np.empty((W, self.count_row // 8), np.int64)
        self.rt.call('glmvx_memcpy_dtoh', m.ctypes.data, self.mail.ptr, m.nbytes, s)
        torch.cuda.current_stream(self.device).synchronize()
        code = C.c_int32(0)
        self.rt.call('glmvx_check_device_error', C.byref(code))
        if code.value:
            raise RuntimeError('peer exchange: a rank did not deliver its counts in time')
        self.M = m[:, :W].copy()  # M[s, d]: rows rank s sends to rank d
        return self.M[:, self.rank].copy()

    def rows(self, send, send_counts, recv_counts):
        W, r = self.world, self.rank
        S, dst_rows, total = peer_layout(self.M, send_counts, r)
        if self.call >= self.REGIONS:
            raise RuntimeError('more than three rows() exchanges after one counts()')
        region, self.call = self.call, self.call + 1
        n = int(send.shape[0])
        rb = int(np.prod(send.shape[1:], dtype=np.int64)) * send.element_size()  # bytes per row
        rb16 = _pad16(max(rb, 1))
        if rb16 > self.row_cap or total > self.max_rows:
            raise ValueError('peer exchange: more rows or wider rows than the mailbox holds')
        off = self.data_off + region * self.region_bytes
        if n:
            flat = send.contiguous().view(torch.uint8).reshape(n, rb)
            if rb16 != rb:
                padded = torch.zeros((n, rb16), dtype=torch.uint8, device=send.device)
                padded[:, :rb] = flat
                flat = padded
            dst = [self.base[d] + off for d in range(W)]
            self.rt.call('glmvx_p2p_scatter', flat.data_ptr(), rb16, self._ptrs(dst),
                         self._i64(np.asarray(send_counts, np.int64)), self._i64(dst_rows), W, self._stream())
        self._exchange_done(region + 1)
        recv = self.view[off:off + total * rb16].view(total, rb16)[:, :rb].contiguous()
        return recv.view(send.dtype).reshape((total,) + tuple(send.shape[1:]))

    def close(self):
        for d, p in enumerate(getattr(self, 'base', [])):
            if d != self.rank and p:
                self.rt.call('glmvx_ipc_close', p)
        self.base = []
        for b in ('stage', 'mail'):
            if getattr(self, b, None) is not None:
                getattr(self, b).close()


def ep_step(x, ids, wts, per_rank, exchange, ops):
    """One expert-parallel layer step for this rank's token rows.

    x: tensor [T, hidden] on the exchange device; ids/wts: host arrays [T, k]
    from the (replicated) router.  `ops` supplies the compute on that device:
      gather(x, idx_int32) -> x[idx]            (tensors)
      experts(rows, local_ids_int32) -> out     (this rank's experts)
      shared(x) -> rows or None                 (shared expert)
      combine(pair_out, comb, combw, shared) -> y
    Returns y [T, hidden]."""
    ids = np.asarray(ids)
    T, k = ids.shape
    order, send_counts = dispatch_plan(ids, per_rank, exchange.world)
    recv_counts = exchange.counts(send_counts)
    flat = ids.reshape(-1)[order]
    local_ids = (flat - (flat // per_rank) * per_rank).astype(np.int32)
    token_of_pair = (order // k).astype(np.int32)
    send_rows = ops.gather(x, token_of_pair)
    recv_rows = exchange.rows(send_rows, send_counts, recv_counts)
    recv_ids = exchange.rows(torch.as_tensor(local_ids, device=exchange.device), send_counts, recv_counts)
    out_rows = ops.experts(recv_rows, recv_ids)
    pair_out = exchange.rows(out_rows, recv_counts, send_counts)
    comb, combw = combine_plan(ids, wts, order)
    return ops.combine(pair_out, comb, combw, ops.shared(x))


class _CudaOps:
    """ep_step compute on the CUDA library, on torch's current stream."""

    def __init__(self, layer):
        self.layer = layer

    def _stream(self):
        return torch.cuda.current_stream().cuda_stream

    def gather(self, x, idx):
        lay = self.layer
        idx_d = torch.as_tensor(idx, device=x.device)
        out = torch.empty((len(idx), lay.hidden), dtype=torch.float32, device=x.device)
        lay._check(lay.lib.glmvx_gather_rows(out.data_ptr(), x.data_ptr(), idx_d.data_ptr(), len(idx), lay.hidden,
                                             self._stream()), 'glmvx_gather_rows')
        return out

    def _run_experts(self, rows, ids, experts, stacks):
        lay = self.layer
        n = rows.shape[0]
        out = torch.empty((n, lay.hidden), dtype=torch.float32, device=rows.device)
        if n == 0:
            return out
        need = int(lay.lib.glmvx_moe_workspace_bytes(n, lay.hidden, lay.inter, experts, 1, 0))
        ws = torch.empty(need, dtype=torch.uint8, device=rows.device)
        lay._check(lay.lib.glmvx_moe_experts(out.data_ptr(), rows.data_ptr(), ids.data_ptr(), n, lay.hidden,
                                             lay.inter, experts, lay.kind, *stacks, ws.data_ptr(), need,
                                             self._stream()), 'glmvx_moe_experts')
        return out

    def experts(self, rows, ids):
        lay = self.layer
        return self._run_experts(rows, ids, lay.local_experts, (lay.gate, lay.up, lay.down))

    def shared(self, x):
        lay = self.layer
        if lay.shared[0] is None:
            return None
        zeros = torch.zeros(x.shape[0], dtype=torch.int32, device=x.device)
        return self._run_experts(x, zeros, 1, lay.shared)

    def combine(self, pair_out, comb, combw, shared):
        lay = self.layer
        T, k = comb.shape
        y = torch.empty((T, lay.hidden), dtype=torch.float32, device=pair_out.device)
        comb_d = torch.as_tensor(comb, device=pair_out.device)
        combw_d = torch.as_tensor(combw, device=pair_out.device)
        lay._check(lay.lib.glmvx_moe_combine(y.data_ptr(), pair_out.data_ptr(), comb_d.data_ptr(),
                                             combw_d.data_ptr(), shared.data_ptr() if shared is not None else None,
                                             T, k, lay.hidden, self._stream()), 'glmvx_moe_combine')
        return y


class ExpertParallelMoE:
    """The config-2 MoE layer with its routed experts sharded over the ranks
    of an NCCL process group (one GPU per rank, torch.cuda device already
    selected).  `gate`/`up`/`down` hold only this rank's experts
    ([experts/world][rows][row_bytes] packed GGML bytes); the router, its
    bias and the shared expert are the full, replicated arrays."""

    def __init__(self, router_w, router_bias, kind, gate, up, down, experts, hidden, inter, top_k, scale,
                 shared=None, group=None, exchange='nccl', max_tokens=64):
        from . import runtime as rt
        from kernels.packed import LAYOUTS
        self.rt, self.lib = rt, rt.library()
        self.kind, self.experts, self.hidden, self.inter = int(kind), int(experts), int(hidden), int(inter)
        self.top_k, self.scale = int(top_k), float(scale)
        self.exchange = Exchange(group, torch.device('cuda', torch.cuda.current_device()))
        # The library keeps its own CUDA runtime state: select the same device.
        rt.call('glmvx_set_device', torch.cuda.current_device())
        self.per_rank = experts_per_rank(self.experts, self.exchange.world)
        if exchange == 'peer':  # rows over NVLink peer stores instead of NCCL (PeerExchange)
            self.exchange = PeerExchange(group, self.exchange.device, self.exchange.world * max_tokens * self.top_k,
                                         4 * self.hidden)
        elif exchange != 'nccl':
            raise ValueError("exchange must be 'nccl' or 'peer'")
        self.local_experts = self.per_rank
        block, size, _ = LAYOUTS[self.kind]
        one = self.inter * (self.hidden // block) * size
        for name, arr in (('gate', gate), ('up', up), ('down', down)):
            if np.asarray(arr).nbytes != self.per_rank * one:
                raise ValueError(f'{name} must hold this rank\'s {self.per_rank} experts')
        dev = self.exchange.device

        def upload(a):
            a = np.ascontiguousarray(a)
            return torch.from_numpy(a.reshape(-1).view(np.uint8).copy()).to(dev)

        self._keep = [upload(np.asarray(router_w, np.float32)), upload(np.asarray(router_bias, np.float32)),
                      upload(gate), upload(up), upload(down)]
        self.router_w, self.router_bias, self.gate, self.up, self.down = (t.data_ptr() for t in self._keep)
        if shared is not None:
            sh = [upload(a) for a in shared]
            self._keep += sh
            self.shared = tuple(t.data_ptr() for t in sh)
        else:
            self.shared = (None, None, None)
        self.ops = _CudaOps(self)

    def _check(self, code, name):
        self.rt.check(self.lib, code, name)

    def close(self):
        """Unmap the peers' mailboxes and free this rank's (peer exchange);
        call on every rank after its last step has finished."""
        if hasattr(self.exchange, 'close'):
            self.exchange.close()

    def route(self, x):
        """Replicated router on this rank's rows -> host ids, weights."""
        T = x.shape[0]
        stream = torch.cuda.current_stream().cuda_stream
        logits = torch.empty((T, self.experts), dtype=torch.float32, device=x.device)
        ids = torch.empty((T, self.top_k), dtype=torch.int32, device=x.device)
        wts = torch.empty((T, self.top_k), dtype=torch.float32, device=x.device)
        self._check(self.lib.glmvx_matmul_nt(logits.data_ptr(), x.data_ptr(), self.router_w, T, self.experts,
                                             self.hidden, stream), 'glmvx_matmul_nt')
        self._check(self.lib.glmvx_router(ids.data_ptr(), wts.data_ptr(), logits.data_ptr(), self.router_bias, T,
                                          self.experts, self.top_k, self.scale, stream), 'glmvx_router')
        return ids.cpu().numpy(), wts.cpu().numpy()

    def forward(self, x):
        """x: host float32 [T, hidden] -> (y, ids, weights) on the host."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        if x.ndim != 2 or x.shape[1] != self.hidden:
            raise ValueError('MoE input must be [tokens, hidden]')
        if not np.isfinite(x).all():
            raise ValueError('MoE input must be finite')
        self.rt.call('glmvx_set_device', self.exchange.device.index)
        xd = torch.from_numpy(x).to(self.exchange.device)
        ids, wts = self.route(xd)
        y = ep_step(xd, ids, wts, self.per_rank, self.exchange, self.ops)
        y = y.cpu().numpy()
        if not np.isfinite(y).all():
            raise ValueError('nonfinite MoE output')
        return y, ids, wts
