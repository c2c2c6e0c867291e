"""Expert-parallel MoE protocol on CPU (tests/ep_model.py, the host model of
the device protocol in csrc/ep.cu): dispatch/combine planning, the device
mailbox plan, and a full layer step over 2- and 4-rank gloo groups with the
CPU oracle as the expert compute, which must reproduce the single-process
reference layer (glm_vx/model.py:289-324) bit for bit."""
import os
import socket

import numpy as np
import pytest

from kernels.packed import LAYOUTS


def test_dispatch_plan_groups_pairs_by_owner():
    from ep_model import dispatch_plan
    ids = np.array([[5, 0, 7], [2, 6, 1]], np.int32)  # 8 experts over 2 ranks: 0-3 on rank 0
    order, counts = dispatch_plan(ids, 4, 2)
    assert counts.tolist() == [3, 3]
    assert order.tolist() == [1, 3, 5, 0, 2, 4]  # rank 0 pairs in (token, slot) order, then rank 1
    with pytest.raises(ValueError, match='sharded range'):
        dispatch_plan(np.array([[8]]), 4, 2)


def test_combine_plan_is_ascending_expert_order():
    from ep_model import combine_plan, dispatch_plan
    ids = np.array([[5, 0, 7], [2, 6, 1]], np.int32)
    wts = np.array([[0.5, 0.25, 0.125], [1.0, 2.0, 3.0]], np.float32)
    order, _ = dispatch_plan(ids, 4, 2)
    comb, combw = combine_plan(ids, wts, order)
    sent = order[comb]  # flattened pair index behind each combine slot
    for t in range(2):
        experts = ids.reshape(-1)[sent[t]]
        assert experts.tolist() == sorted(ids[t].tolist())
        assert combw[t].tolist() == [float(wts[t][list(ids[t]).index(e)]) for e in experts]
    with pytest.raises(ValueError, match='evenly'):
        from ep_model import experts_per_rank
        experts_per_rank(10, 4)


E, H, I, K, T = 8, 512, 256, 2, 3


def _layer():
    from test_gpu_moe import synthetic_layer
    return synthetic_layer(E, H, I, kind=19, seed=41)


def _tokens(rank):
    return np.random.default_rng(500 + rank).normal(size=(T, H)).astype(np.float32)


class _OracleOps:
    """ep_step compute on the CPU oracle (reference numerics)."""

    def __init__(self, cpu, layer, rank, per_rank):
        self.cpu, self.layer, self.rank, self.per_rank = cpu, layer, rank, per_rank
        block, size, _ = LAYOUTS[19]
        self.gu, self.dn = I * (H // block) * size, H * (I // block) * size

    def _mlp(self, g, u, d, v):
        cpu = self.cpu
        gate = cpu.packed_matvec(g, 19, (I, H), v)
        up = cpu.packed_matvec(u, 19, (I, H), v)
        return cpu.packed_matvec(d, 19, (H, I), cpu.swiglu(gate, up))

    def gather(self, x, idx):
        import torch
        return x[torch.as_tensor(idx, dtype=torch.long)]

    def experts(self, rows, ids):
        import torch
        lay, out = self.layer, []
        for v, j in zip(rows.numpy(), ids.numpy()):
            e = self.rank * self.per_rank + int(j)
            out.append(self._mlp(lay['gate'][e * self.gu:(e + 1) * self.gu], lay['up'][e * self.gu:(e + 1) * self.gu],
                                 lay['down'][e * self.dn:(e + 1) * self.dn], v))
        return torch.from_numpy(np.stack(out) if out else np.empty((0, H), np.float32))

    def shared(self, x):
        import torch
        return torch.from_numpy(np.stack([self._mlp(*self.layer['shared'], v) for v in x.numpy()]))

    def combine(self, pair_out, comb, combw, shared):
        import torch
        p, s = pair_out.numpy(), shared.numpy()
        y = np.zeros((comb.shape[0], H), np.float32)
        for t in range(comb.shape[0]):
            for i in range(comb.shape[1]):
                y[t] += p[comb[t, i]] * combw[t, i]
            y[t] += s[t]
        return torch.from_numpy(y)


def _rank_main(rank, world, port, out_dir):
    import torch.distributed as dist
    import torch
    os.environ['MASTER_ADDR'], os.environ['MASTER_PORT'] = '127.0.0.1', str(port)
    from datetime import timedelta
    dist.init_process_group('gloo', rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        from oracle import loader
        from kernels.backend import VxBackend
        from ep_model import Exchange, ep_step
        cpu = VxBackend(str(loader.serial()))
        layer, x = _layer(), _tokens(rank)
        ids, wts = [], []
        for v in x:
            i, w = cpu.route(cpu.matvec(layer['router'], v), layer['bias'], K, 2.5)
            ids.append(i)
            wts.append(w)
        ids, wts = np.array(ids, np.int32), np.array(wts, np.float32)
        ex = Exchange(None, 'cpu')
        y = ep_step(torch.from_numpy(x), ids, wts, E // world, ex, _OracleOps(cpu, layer, rank, E // world))
        np.savez(os.path.join(out_dir, f'rank{rank}.npz'), y=y.numpy(), ids=ids)
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(('127.0.0.1', 0))
        return s.getsockname()[1]


@pytest.mark.parametrize('world', [2, 4])
def test_ep_step_over_gloo_matches_reference(tmp_path, oracle, world):
    import torch.multiprocessing as mp
    from test_gpu_moe import reference_ffn
    mp.spawn(_rank_main, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    layer = _layer()
    for rank in range(world):
        got = np.load(tmp_path / f'rank{rank}.npz')
        want, want_ids = reference_ffn(oracle, layer, _tokens(rank), E, H, I, K, 2.5)
        assert got['ids'].tolist() == want_ids.tolist()
        assert got['y'].tobytes() == want.tobytes()


def test_mailbox_plan_matches_host_plan():
    """The device dispatch (ep_dispatch_kernel) places pair a of destination d
    at position pos[a] of d's region for this sender, in (token, slot) order,
    and the combine reads owner * cap + pos in ascending expert id: the same
    pairs, order and combine sequence as the host plan (all_to_all order)."""
    from ep_model import combine_plan, dispatch_plan, mailbox_plan
    rng = np.random.default_rng(9)
    for world, experts, k, T in ((1, 8, 2, 3), (2, 16, 4, 5), (4, 256, 8, 32), (8, 256, 8, 32)):
        per = experts // world
        ids = np.stack([rng.choice(experts, size=k, replace=False) for _ in range(T)]).astype(np.int32)
        wts = rng.random((T, k)).astype(np.float32)
        cap = T * k
        dest, pos, counts, rows = mailbox_plan(ids, per, world, cap)
        order, host_counts = dispatch_plan(ids, per, world)
        assert counts.tolist() == host_counts.tolist()
        starts = np.concatenate([[0], np.cumsum(host_counts)[:-1]])
        # position in the all_to_all send order = start of the destination + position in it
        assert (starts[dest] + pos)[order].tolist() == list(range(T * k))
        comb, _ = combine_plan(ids, wts, order)
        # the same pair behind every combine slot
        flat_of_row = {int(dest[a] * cap + pos[a]): a for a in range(T * k)}
        assert [[flat_of_row[int(r)] for r in row] for row in rows] == order[comb].tolist()
