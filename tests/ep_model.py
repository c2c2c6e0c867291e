"""Test infrastructure: a host model of the expert-parallel protocol.

The product runs the protocol on the device (glm-vx_b200/csrc/ep.cu,
gpu/ep.py): every (token, slot) pair goes to the rank owning its expert
(expert e on rank e // (experts / world)), grouped by destination in
(token, slot) order; the owner computes; each token sums its pair outputs
in ascending expert id and adds the shared expert last
(glm_vx/model.py:289-324).  This module restates that plan on the host and
runs it over a torch.distributed (gloo) group with the CPU oracle as the
expert compute, so the CPU tests check the protocol's order and reduction
semantics against the single-process reference without a GPU.
"""
import numpy as np

import torch
import torch.distributed as dist


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




def mailbox_plan(ids, per_rank, world, cap):
    """The device dispatch plan (ep_dispatch_kernel): for every pair a = t*k+j
    its destination rank and its position among the pairs to that rank, and
    per token the rows of the rank's return region (owner * cap + position)
    in ascending expert id -- what the combine reads."""
    ids = np.asarray(ids)
    T, k = ids.shape
    flat = ids.reshape(-1)
    dest = flat // per_rank
    pos = np.zeros(T * k, np.int64)
    run = np.zeros(world, np.int64)
    for a in range(T * k):
        pos[a] = run[dest[a]]
        run[dest[a]] += 1
    rows = (dest * cap + pos).reshape(T, k)
    srt = np.argsort(ids, axis=1, kind='stable')
    return dest, pos, run, rows[np.arange(T)[:, None], srt]
