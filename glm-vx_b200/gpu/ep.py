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
                 shared=None, group=None):
        from . import runtime as rt
        from kernels.packed import LAYOUTS
        self.rt, self.lib = rt, rt.library()
        self.kind, self.experts, self.hidden, self.inter = int(kind), int(experts), int(hidden), int(inter)
        self.top_k, self.scale = int(top_k), float(scale)
        self.exchange = Exchange(group, torch.device('cuda', torch.cuda.current_device()))
        # The library keeps its own CUDA runtime state: select the same device.
        rt.call('glmvx_set_device', torch.cuda.current_device())
        self.per_rank = experts_per_rank(self.experts, self.exchange.world)
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
