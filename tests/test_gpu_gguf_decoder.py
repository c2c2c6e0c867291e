"""The resident decoder loading a split GLM-DSA GGUF checkpoint
(gpu/gguf_source.py) against the reference model reading the same files
through its own GGUF loader (glm_vx/gguf_checkpoint.py GGUFCheckpoint,
packed weights on the reference VxBackend over the CPU oracle).  Same bar as
the decoder parity test: identical greedy tokens, logits within 1e-5."""
import numpy as np
import pytest

import refmodel

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not refmodel.available(), reason='reference not installed in baseline/_ref')]

PROMPTS = [[37, 401, 5, 260, 118, 77], [255, 0, 511, 64, 128, 256]]
NEW_TOKENS = 6


def test_decoder_from_split_gguf_matches_reference_gguf(gpu_backend, tmp_path):
    import gguf_fixture
    from oracle import loader
    refmodel.ref_glm_vx()
    from glm_vx.gguf_checkpoint import GGUFCheckpoint
    from glm_vx.model import GlmMoeDsaModel
    from gpu.decoder import ResidentDecoder
    from gpu.gguf_source import GGUFSource
    config = refmodel.dropin_config(layers=3, width=256)
    ckpt = refmodel.PackedCheckpoint(config, seed=5)
    paths = gguf_fixture.write_checkpoint(ckpt, config, tmp_path / 'glm.gguf', split_max_tensors=16)
    assert len(paths) > 2
    ref_ckpt = GGUFCheckpoint(str(paths[0]), config)
    try:
        model = GlmMoeDsaModel(config, ref_ckpt, refmodel.ref_vx_backend(loader.parallel()), packed_weights=True)
        runs = [refmodel.greedy(model, p, NEW_TOKENS, grouped_prefill=False) for p in PROMPTS]
    finally:
        ref_ckpt.close()
    src = GGUFSource(paths[1], config, gpu_backend)  # any file of the set opens it
    dec = ResidentDecoder(gpu_backend, config, src, batch=len(PROMPTS), capacity=24)
    try:
        tokens, logits = dec.generate(np.array(PROMPTS), NEW_TOKENS, with_logits=True)
        for b, (want_tokens, want_logits) in enumerate(runs):
            assert tokens[b].tolist() == want_tokens, b
            for s in range(NEW_TOKENS):
                err = np.linalg.norm(logits[b, s] - want_logits[s]) / np.linalg.norm(want_logits[s])
                assert err <= 1e-5, (b, s, err)
    finally:
        dec.close()
        src.close()
