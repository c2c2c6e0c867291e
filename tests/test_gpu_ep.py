"""Expert-parallel MoE layer (csrc/ep.cu, gpu/ep.py) on the GPU.

A token's arithmetic in the expert-parallel step is the single-GPU layer's
(the same prepared rows, job kernels and ascending-expert-id combine), so
every rank's output must equal gpu.moe.MoELayer on the same rows BIT FOR
BIT, at any number of ranks; and MoELayer is pinned to the reference's
sparse feed-forward (glm_vx/model.py:289-324) on the CPU oracle.

On one GPU the ranks are emulated in one process (`emulated_ranks`: the
mailboxes are plain device pointers and the phases run rank by rank on one
stream, so every device wait is already satisfied when it runs).  With two
GPUs the real thing runs: one process per GPU, mailboxes mapped through
CUDA IPC handles swapped by a file bootstrap, one captured graph per step."""
import multiprocessing as mp
import os

import numpy as np
import pytest

from helpers import RTOL
from test_gpu_moe import reference_ffn, synthetic_layer

pytestmark = pytest.mark.gpu

E, H, I, K = 16, 2048, 2048, 4


def _moe(backend, layer, experts, hidden, inter, k):
    from gpu.moe import MoELayer
    return MoELayer(backend, layer['router'], layer['bias'], 19, layer['gate'], layer['up'], layer['down'], hidden,
                    inter, k, 2.5, shared=layer['shared'])


@pytest.mark.parametrize('world,T', [(1, 5), (2, 5), (4, 3), (8, 2), (2, 17), (4, 9)])
def test_emulated_ranks_match_single_gpu_layer(gpu_backend, world, T):
    from gpu.ep import emulated_forward, emulated_ranks
    layer = synthetic_layer(E, H, I, kind=19, seed=70 + world)
    xs = [np.random.default_rng(100 * world + r).normal(size=(T, H)).astype(np.float32) for r in range(world)]
    ranks = emulated_ranks(gpu_backend, world, layer, 19, H, I, K, 2.5, max_tokens=max(T, 8))
    moe = _moe(gpu_backend, layer, E, H, I, K)
    try:
        for step in range(2):  # the second step reuses every mailbox
            got = emulated_forward(ranks, xs)
            for r in range(world):
                y, ids, w = moe.forward(xs[r])
                assert got[r][1].tolist() == ids.tolist()
                assert got[r][2].tobytes() == w.tobytes()
                assert got[r][0].tobytes() == y.tobytes(), (step, r)
    finally:
        for lay in ranks:
            lay.close()
        moe.close()


def test_emulated_ranks_against_oracle(gpu_backend, oracle):
    from gpu.ep import emulated_forward, emulated_ranks
    layer = synthetic_layer(E, H, I, kind=19, seed=71)
    xs = [np.random.default_rng(31 + r).normal(size=(4, H)).astype(np.float32) for r in range(2)]
    ranks = emulated_ranks(gpu_backend, 2, layer, 19, H, I, K, 2.5, max_tokens=8)
    try:
        got = emulated_forward(ranks, xs)
    finally:
        for lay in ranks:
            lay.close()
    for r in range(2):
        want, want_ids = reference_ffn(oracle, layer, xs[r], E, H, I, K, 2.5)
        assert got[r][1].tolist() == want_ids.tolist()
        assert np.linalg.norm(got[r][0] - want) / np.linalg.norm(want) <= RTOL


def test_emulated_ranks_uneven_tokens_and_idle_rank(gpu_backend):
    """Ranks with different token counts, one with none (it still takes part
    in the step: its experts serve the others and it signals its returns)."""
    from gpu.ep import emulated_forward, emulated_ranks
    layer = synthetic_layer(E, H, I, kind=19, seed=72)
    counts = [6, 0, 1, 3]
    xs = [np.random.default_rng(40 + r).normal(size=(n, H)).astype(np.float32) for r, n in enumerate(counts)]
    ranks = emulated_ranks(gpu_backend, 4, layer, 19, H, I, K, 2.5, max_tokens=8)
    moe = _moe(gpu_backend, layer, E, H, I, K)
    try:
        got = emulated_forward(ranks, xs)
        for r, n in enumerate(counts):
            assert got[r][0].shape == (n, H)
            if n:
                assert got[r][0].tobytes() == moe.forward(xs[r])[0].tobytes()
    finally:
        for lay in ranks:
            lay.close()
        moe.close()


def test_config2_full_width_eight_emulated_ranks(gpu_backend):
    """The benchmarked layer (256 IQ1_S experts + shared, hidden 6144,
    inter 2048, top-8) split over 8 ranks of 32 experts, 32 tokens per rank:
    every rank's output equals the full single-GPU layer's bit for bit."""
    from gpu.ep import emulated_forward, emulated_ranks
    layer = synthetic_layer(256, 6144, 2048, kind=19, seed=2)
    xs = [np.random.default_rng(300 + r).normal(size=(32, 6144)).astype(np.float32) for r in range(8)]
    ranks = emulated_ranks(gpu_backend, 8, layer, 19, 6144, 2048, 8, 2.5, max_tokens=32)
    try:
        got = emulated_forward(ranks, xs)
    finally:
        for lay in ranks:
            lay.close()
    moe = _moe(gpu_backend, layer, 256, 6144, 2048, 8)
    try:
        for r in range(8):
            y, ids, _ = moe.forward(xs[r])
            assert got[r][1].tolist() == ids.tolist()
            assert got[r][0].tobytes() == y.tobytes(), r
    finally:
        moe.close()


def test_single_rank_graph_step(gpu_backend):
    """world = 1 through the public forward (pinned I/O, one captured graph
    per step): equal to MoELayer; zero tokens is a valid step."""
    from gpu.ep import ExpertParallelLayer
    layer = synthetic_layer(E, H, I, kind=19, seed=73)
    lay = ExpertParallelLayer(gpu_backend, 0, 1, layer['router'], layer['bias'], 19, layer['gate'], layer['up'],
                              layer['down'], E, H, I, K, 2.5, shared=layer['shared'], max_tokens=8)
    lay.connect([lay.mailbox()[0]])
    moe = _moe(gpu_backend, layer, E, H, I, K)
    try:
        x = np.random.default_rng(3).normal(size=(7, H)).astype(np.float32)
        for _ in range(3):
            y, ids, _ = lay.forward(x)
            want, want_ids, _ = moe.forward(x)
            assert ids.tolist() == want_ids.tolist() and y.tobytes() == want.tobytes()
        y0, _, _ = lay.forward(np.empty((0, H), np.float32))
        assert y0.shape == (0, H)
        y, _, _ = lay.forward(x)
        assert y.tobytes() == want.tobytes()
        with pytest.raises(ValueError, match='tokens'):
            lay.forward(np.zeros((9, H), np.float32))
        xb = x.copy()
        xb[1, 5] = np.nan
        with pytest.raises(ValueError, match='finite'):
            lay.forward(xb)
    finally:
        lay.close()
        moe.close()


def test_missing_peer_times_out_without_hanging(gpu_backend):
    """A rank whose peer never dispatches: the owner's bounded wait (2 s)
    gives up, sets the device error word, and the host raises; the context
    stays usable.  (The flag that nothing sets is rank 1's; no kernel is
    broken and nothing is out of bounds.)"""
    from gpu import runtime as rt
    from gpu.ep import emulated_ranks
    layer = synthetic_layer(E, H, I, kind=19, seed=74)
    ranks = emulated_ranks(gpu_backend, 2, layer, 19, H, I, K, 2.5, max_tokens=4)
    x = np.random.default_rng(1).normal(size=(2, H)).astype(np.float32)
    xd, yd = rt.DeviceBuffer(x.nbytes), rt.DeviceBuffer(x.nbytes)
    try:
        xd.upload(x, gpu_backend.stream.handle)
        ranks[0].dispatch(xd.ptr, 2)
        ranks[0].run_experts(2)  # waits for rank 1, which never dispatched
        gpu_backend.stream.synchronize()
        with pytest.raises(Exception, match='device'):
            gpu_backend.device.check_device_error()
        gpu_backend.device.check_device_error()  # cleared: the device keeps working
    finally:
        gpu_backend.stream.synchronize()
        for lay in ranks:
            lay.close()
        xd.close()
        yd.close()
    moe = _moe(gpu_backend, layer, E, H, I, K)
    try:
        y, _, _ = moe.forward(x)
        assert np.isfinite(y).all()
    finally:
        moe.close()


def _gpus():
    from gpu import runtime
    try:
        return runtime.device_count()
    except Exception:
        return 0


def _rank_main(rank, world, boot_dir, out_dir):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [root, os.path.join(root, 'glm-vx_b200'), os.path.join(root, 'tests')]
    from gpu.backend import GPUBackend
    from gpu.ep import ExpertParallelLayer, FileBootstrap, split_layer
    backend = GPUBackend(rank)
    boot = FileBootstrap(boot_dir, rank, world)
    layer = synthetic_layer(E, H, I, kind=19, seed=77)
    g, u, d = split_layer(layer, world, rank)
    lay = ExpertParallelLayer(backend, rank, world, layer['router'], layer['bias'], 19, g, u, d, E, H, I, K, 2.5,
                              shared=layer['shared'], max_tokens=8)
    lay.connect_ipc(boot.allgather)
    x = np.random.default_rng(900 + rank).normal(size=(5, H)).astype(np.float32)
    y, ids, _ = lay.forward(x)
    y2, _, _ = lay.forward(x)
    lay.close(barrier=boot.barrier)
    backend.close()
    np.savez(os.path.join(out_dir, f'rank{rank}.npz'), x=x, y=y, y2=y2, ids=ids)


@pytest.mark.skipif(_gpus() < 2, reason='needs two GPUs')
def test_two_gpu_processes_over_ipc_mailboxes(tmp_path, oracle):
    ctx = mp.get_context('spawn')
    procs = [ctx.Process(target=_rank_main, args=(r, 2, str(tmp_path / 'boot'), str(tmp_path))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        assert p.exitcode == 0
    layer = synthetic_layer(E, H, I, kind=19, seed=77)
    for r in range(2):
        got = np.load(tmp_path / f'rank{r}.npz')
        want, want_ids = reference_ffn(oracle, layer, got['x'], E, H, I, K, 2.5)
        assert got['ids'].tolist() == want_ids.tolist()
        assert np.linalg.norm(got['y'] - want) / np.linalg.norm(want) <= RTOL
        assert got['y2'].tobytes() == got['y'].tobytes()
