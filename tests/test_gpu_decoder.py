"""Resident batched greedy decode (gpu/decoder.py) against the reference
model's own greedy decode on the CPU oracle.

The reference (glm_vx/model.py GlmMoeDsaModel, installed unmodified in
baseline/_ref) decodes each prompt alone, one token per call, through the
reference VxBackend over the oracle library; the resident decoder decodes
all of them in one batch on the B200, one captured graph per step, with the
next token chosen on the device.  Same packed weights (IQ1_S experts and
dense MLP, Q4_K / Q8_0 attention projections, Q8_0 lm_head, F32 router,
indexer head weights and kv_b), the reference's tiny config widened to
block-aligned sizes (4 layers: dense + sparse, full + shared DSA indexers).
Bar: the greedy token streams are identical, every sampled step's logits
within 1e-5 normwise of the reference's."""
import numpy as np
import pytest

import refmodel

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not refmodel.available(), reason='reference not installed in baseline/_ref')]

PROMPTS = [[37, 401, 5, 260, 118, 77], [3, 3, 3, 500, 12, 9], [255, 0, 511, 64, 128, 256]]
NEW_TOKENS = 8


@pytest.fixture(scope='module', params=[256, 2048], ids=['w256', 'w2048'])
def reference_runs(request):
    """Width 256 runs the CUDA-core expert jobs, 2048 the tensor-core ones."""
    refmodel.ref_glm_vx()
    from glm_vx.model import GlmMoeDsaModel
    from oracle import loader
    config = refmodel.dropin_config(width=request.param)
    ckpt = refmodel.PackedCheckpoint(config, seed=1)
    model = GlmMoeDsaModel(config, ckpt, refmodel.ref_vx_backend(loader.parallel()), packed_weights=True)
    runs = [refmodel.greedy(model, p, NEW_TOKENS, grouped_prefill=False) for p in PROMPTS]
    return config, ckpt, runs


def test_resident_decoder_greedy_matches_reference(gpu_backend, reference_runs):
    from gpu.decoder import ResidentDecoder
    config, ckpt, runs = reference_runs
    dec = ResidentDecoder(gpu_backend, config, ckpt, batch=len(PROMPTS), capacity=32)
    try:
        tokens, logits = dec.generate(np.array(PROMPTS), NEW_TOKENS, with_logits=True)
        for b, (want_tokens, want_logits) in enumerate(runs):
            assert tokens[b].tolist() == want_tokens, b
            for s in range(NEW_TOKENS):
                got, want = logits[b, s], want_logits[s]
                err = np.linalg.norm(got - want) / np.linalg.norm(want)
                assert err <= 1e-5, (b, s, err)
        # the cache keeps going: a second generate() restarts from empty caches
        tokens2, _ = dec.generate(np.array(PROMPTS), NEW_TOKENS)
        assert tokens2.tolist() == tokens.tolist()
    finally:
        dec.close()


def test_resident_decoder_single_sequence_equals_batch(gpu_backend, reference_runs):
    """A sequence decodes the same alone as inside a batch."""
    from gpu.decoder import ResidentDecoder
    config, ckpt, runs = reference_runs
    dec = ResidentDecoder(gpu_backend, config, ckpt, batch=1, capacity=32)
    try:
        tokens, _ = dec.generate(np.array(PROMPTS[1:2]), NEW_TOKENS)
        assert tokens[0].tolist() == runs[1][0]
    finally:
        dec.close()


def test_synthetic_config4_shapes_run(gpu_backend):
    """BASELINE config-4 widths (hidden 6144, 64 heads, rank 512, indexer
    32 x 128 top-2048, 256 IQ1_S experts + shared, vocab 154880), two layers
    (dense + sparse) of device-generated weights, 4 sequences over caches of
    2100 synthetic rows: steps run, logits are finite, tokens are in the
    vocabulary and the same seed gives the same tokens."""
    from gpu.decoder import ResidentDecoder, SyntheticWeights
    import bench
    cfg = dict(bench.CONFIG4, first_k_dense_replace=1)
    outs = []
    for _ in range(2):
        dec = ResidentDecoder(gpu_backend, cfg, SyntheticWeights(cfg, seed=5), batch=4, capacity=2112, layers=2)
        try:
            dec.fill_caches(2100)
            dec.set_tokens([1, 2, 3, 4])
            toks = []
            for _ in range(3):
                dec.step()
                toks.append(dec.read_tokens())
            logits = dec.read_logits()
            dec.check()
            assert np.isfinite(logits).all()
            assert all(0 <= t < cfg['vocab_size'] for row in toks for t in row)
            outs.append(np.stack(toks))
        finally:
            dec.close()
    assert outs[0].tolist() == outs[1].tolist()


EP_PROMPTS = PROMPTS + [[7, 8, 9, 10, 11, 12]]


def _gpus():
    from gpu import runtime
    try:
        return runtime.device_count()
    except Exception:
        return 0


def _ep_rank_main(rank, world, boot_dir, out_path, gguf_path=None):
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parents[1]
    sys.path[:0] = [str(root), str(root / 'glm-vx_b200'), str(root / 'tests')]
    import refmodel as R
    from gpu.backend import GPUBackend
    from gpu.decoder import ResidentDecoder, expert_parallel_moe
    from gpu.ep import FileBootstrap
    backend = GPUBackend(rank)
    boot = FileBootstrap(boot_dir, rank, world)
    config = R.dropin_config(width=2048)
    if gguf_path:  # this rank's experts read straight from the split GGUF files
        from gpu.gguf_source import GGUFSource
        ckpt = GGUFSource(gguf_path, config, backend)
    else:
        ckpt = R.PackedCheckpoint(config, seed=1)
    per = len(EP_PROMPTS) // world
    dec = ResidentDecoder(backend, config, ckpt, batch=per, capacity=32,
                          moe_layer_factory=expert_parallel_moe(rank, world, boot.allgather))
    tokens, _ = dec.generate(np.array(EP_PROMPTS[rank * per:(rank + 1) * per]), NEW_TOKENS)
    dec.close(barrier=boot.barrier)
    backend.close()
    np.save(out_path, tokens)


@pytest.mark.skipif(_gpus() < 2, reason='needs two GPUs')
@pytest.mark.parametrize('source', ['packed', 'gguf'])
def test_expert_parallel_decoder_on_two_gpus(tmp_path, source):
    """Two processes, one GPU each: each decodes two of the four prompts
    (data-parallel attention) while the sparse layers' experts are split
    between the GPUs (gpu/ep.py over IPC mailboxes); every sequence's greedy
    tokens equal the reference model's own decode on the oracle.  With
    source 'gguf' the ranks load the checkpoint from split GGUF files, each
    uploading only its own experts' slices."""
    import multiprocessing as mp
    refmodel.ref_glm_vx()
    from glm_vx.model import GlmMoeDsaModel
    from oracle import loader
    config = refmodel.dropin_config(width=2048)  # the expert-parallel layer runs the tensor-core widths
    ckpt = refmodel.PackedCheckpoint(config, seed=1)
    model = GlmMoeDsaModel(config, ckpt, refmodel.ref_vx_backend(loader.parallel()), packed_weights=True)
    want = [refmodel.greedy(model, p, NEW_TOKENS, grouped_prefill=False)[0] for p in EP_PROMPTS]
    gguf_path = None
    if source == 'gguf':
        import gguf_fixture
        gguf_path = str(gguf_fixture.write_checkpoint(ckpt, config, tmp_path / 'glm.gguf', split_max_tensors=24)[0])
    ctx = mp.get_context('spawn')
    procs = [ctx.Process(target=_ep_rank_main,
                         args=(r, 2, str(tmp_path / 'boot'), str(tmp_path / f'r{r}.npy'), gguf_path))
             for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        assert p.exitcode == 0
    got = np.concatenate([np.load(tmp_path / f'r{r}.npy') for r in range(2)])
    assert got.tolist() == want


def test_batch_scheduler_matches_reference(gpu_backend, reference_runs):
    """gpu/serving.py over 2 decoder slots, 4 requests (slots reused after a
    request leaves): every greedy request's tokens equal the reference
    model's own greedy decode of its prompt; a sampled request (temperature
    > 0) is reproducible from its seed; status and the reference's
    validation messages hold."""
    from gpu.decoder import ResidentDecoder
    from gpu.serving import BatchScheduler, BusyError, collect
    config, ckpt, runs = reference_runs
    dec = ResidentDecoder(gpu_backend, config, ckpt, batch=2, capacity=32)
    sched = BatchScheduler(dec)
    try:
        with pytest.raises(ValueError, match='nonempty'):
            sched.submit([], 4)
        with pytest.raises(ValueError, match='context'):
            sched.submit([1] * 30, 8)
        reqs = [sched.submit(list(PROMPTS[0]), NEW_TOKENS), sched.submit(list(PROMPTS[1]), NEW_TOKENS)]
        with pytest.raises(BusyError):
            sched.submit([1, 2], 2)  # both slots taken
        out = [collect(r) for r in reqs]
        for (tokens, done), want in zip(out, runs[:2]):
            assert done['reason'] == 'length' and done['completion_tokens'] == NEW_TOKENS
            assert tokens == want[0]
        r2 = sched.submit(list(PROMPTS[2]), NEW_TOKENS)
        s1 = sched.submit(list(PROMPTS[0]), 5, temperature=0.7, seed=11)
        t2, _ = collect(r2)
        assert t2 == runs[2][0]
        ts1, _ = collect(s1)
        s2 = sched.submit(list(PROMPTS[0]), 5, temperature=0.7, seed=11)
        ts2, _ = collect(s2)
        assert ts1 == ts2 and len(ts1) == 5
        assert sched.status()['error'] is None and sched.status()['active_requests'] == 0
    finally:
        sched.close()
        dec.check()
        dec.close()
