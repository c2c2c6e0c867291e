"""Expert-parallel MoE layer (gpu/ep.py ExpertParallelMoE) on 2 GPUs, rows
exchanged over NCCL or over the peer-memory mailboxes (PeerExchange,
csrc/p2p.cu), against the single-process reference layer
(glm_vx/model.py:289-324) on the CPU oracle.  Runs as child processes, one per GPU; skipped when the
box has fewer than two GPUs."""
import os
import socket

import numpy as np
import pytest

from helpers import RTOL

pytestmark = pytest.mark.gpu

E, H, I, K, T = 16, 2048, 2048, 4, 5


def _gpus():
    try:
        import torch
        return torch.cuda.device_count()
    except Exception:
        return 0


def _layer():
    from test_gpu_moe import synthetic_layer
    return synthetic_layer(E, H, I, kind=19, seed=77)


def _tokens(rank):
    return np.random.default_rng(900 + rank).normal(size=(T, H)).astype(np.float32)


def _rank_main(rank, world, port, out_dir, exchange='nccl'):
    os.environ.update(MASTER_ADDR='127.0.0.1', MASTER_PORT=str(port), NCCL_NVLS_ENABLE='0')
    import torch
    import torch.distributed as dist
    from datetime import timedelta
    torch.cuda.set_device(rank)
    dist.init_process_group('nccl', rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device('cuda', rank))
    try:
        from gpu.ep import ExpertParallelMoE
        from kernels.packed import LAYOUTS
        block, size, _ = LAYOUTS[19]
        one = I * (H // block) * size
        lay, per = _layer(), E // world
        sl = slice(rank * per * one, (rank + 1) * per * one)
        moe = ExpertParallelMoE(lay['router'], lay['bias'], 19, lay['gate'][sl], lay['up'][sl], lay['down'][sl], E, H,
                                I, K, 2.5, shared=lay['shared'], exchange=exchange)
        y, ids, _ = moe.forward(_tokens(rank))
        y2, _, _ = moe.forward(_tokens(rank))
        torch.cuda.synchronize()
        dist.barrier()  # both ranks' last steps have finished before the mailboxes go
        moe.close()
        np.savez(os.path.join(out_dir, f'rank{rank}.npz'), y=y, y2=y2, ids=ids)
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(('127.0.0.1', 0))
        return s.getsockname()[1]


@pytest.mark.skipif(_gpus() < 2, reason='needs two GPUs')
@pytest.mark.parametrize('exchange', ['nccl', 'peer'])
def test_expert_parallel_layer_on_two_gpus(tmp_path, oracle, exchange):
    """Both transports: NCCL all_to_all and the peer-memory mailboxes."""
    import torch.multiprocessing as mp
    from test_gpu_moe import reference_ffn
    mp.spawn(_rank_main, args=(2, _free_port(), str(tmp_path), exchange), nprocs=2, join=True)
    layer = _layer()
    for rank in range(2):
        got = np.load(tmp_path / f'rank{rank}.npz')
        want, want_ids = reference_ffn(oracle, layer, _tokens(rank), E, H, I, K, 2.5)
        assert got['ids'].tolist() == want_ids.tolist()
        err = np.linalg.norm(got['y'] - want) / np.linalg.norm(want)
        assert err <= RTOL, err
        assert got['y2'].tobytes() == got['y'].tobytes()


def test_peer_exchange_single_rank(tmp_path, oracle):
    """One rank: the peer exchange's scatter / signal / wait kernels run into
    the rank's own mailbox (no IPC mapping), and the layer matches the
    reference as with NCCL."""
    import torch.multiprocessing as mp
    from test_gpu_moe import reference_ffn
    mp.spawn(_rank_main, args=(1, _free_port(), str(tmp_path), 'peer'), nprocs=1, join=True)
    got = np.load(tmp_path / 'rank0.npz')
    want, want_ids = reference_ffn(oracle, _layer(), _tokens(0), E, H, I, K, 2.5)
    assert got['ids'].tolist() == want_ids.tolist()
    err = np.linalg.norm(got['y'] - want) / np.linalg.norm(want)
    assert err <= RTOL, err
    assert got['y2'].tobytes() == got['y'].tobytes()
