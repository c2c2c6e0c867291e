"""The drop-in claim, exercised: the reference's own model class
(glm_vx/model.py GlmMoeDsaModel, installed unmodified in baseline/_ref) with
packed weights (model.py:49-51, 120-127; prefill.py:14-28) runs on this
library two ways and must give the oracle's logits and greedy tokens:

  * the reference's own VxBackend (kernels/backend.py) loading
    libglmvx_cuda.so through the reference C ABI (host pointers, each call
    staged on the B200) -- what setting GLM_VX_LIBRARY does;
  * this package's GPUBackend (`vx-gpu`: resident packed weights, fused
    compressed attention, GPU top-k and index scores).

The checker is the same reference model on the reference VxBackend over the
CPU oracle.  Config: the reference's tiny GLM-MoE-DSA config widened to
block-aligned widths, with IQ1_S experts and dense MLP, Q4_K and Q8_0
attention projections, Q8_0 lm_head and F32 router / indexer head weights.
Bar: 8 greedy tokens identical (argmax-equal stream), every sampled step's
logits within 1e-5 normwise of the oracle's, through the reference's
grouped prefill (packed_linear_batch) and its per-token path."""
import numpy as np
import pytest

import refmodel

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not refmodel.available(), reason='reference not installed in baseline/_ref')]

PROMPT = [37, 401, 5, 260, 118, 77]
NEW_TOKENS = 8


@pytest.fixture(scope='module')
def setup():
    refmodel.ref_glm_vx()
    from glm_vx.model import GlmMoeDsaModel
    from oracle import loader
    config = refmodel.dropin_config()
    ckpt = refmodel.PackedCheckpoint(config, seed=1)
    oracle_model = GlmMoeDsaModel(config, ckpt, refmodel.ref_vx_backend(loader.serial()), packed_weights=True)
    want = {g: refmodel.greedy(oracle_model, PROMPT, NEW_TOKENS, grouped_prefill=g) for g in (True, False)}
    return config, ckpt, want


def _compare(got, want):
    tokens, logits = got
    want_tokens, want_logits = want
    assert tokens == want_tokens
    for a, b in zip(logits, want_logits):
        assert np.linalg.norm(a - b) <= 1e-5 * np.linalg.norm(b), np.linalg.norm(a - b) / np.linalg.norm(b)


@pytest.mark.parametrize('grouped', [True, False])
def test_reference_vxbackend_on_b200_library(setup, cuda_lib, grouped):
    from glm_vx.model import GlmMoeDsaModel
    from gpu.runtime import library_path
    config, ckpt, want = setup
    backend = refmodel.ref_vx_backend(library_path())
    model = GlmMoeDsaModel(config, ckpt, backend, packed_weights=True)
    _compare(refmodel.greedy(model, PROMPT, NEW_TOKENS, grouped_prefill=grouped), want[grouped])


@pytest.mark.parametrize('grouped', [True, False])
def test_reference_model_on_gpubackend(setup, gpu_backend, grouped):
    from glm_vx.model import GlmMoeDsaModel
    config, ckpt, want = setup
    model = GlmMoeDsaModel(config, ckpt, gpu_backend, packed_weights=True)
    _compare(refmodel.greedy(model, PROMPT, NEW_TOKENS, grouped_prefill=grouped), want[grouped])
    gpu_backend.device.check_device_error()
