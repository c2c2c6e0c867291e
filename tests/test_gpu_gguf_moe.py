"""A sparse layer loaded from a GGUF file into HBM (gpu/gguf_moe.py) against
the single-process reference layer (glm_vx/model.py:289-324) on the CPU
oracle over the same bytes; top-k and scale taken from the file."""
import numpy as np
import pytest

from helpers import RTOL

pytestmark = pytest.mark.gpu
gguf = pytest.importorskip('gguf')


def test_moe_layer_from_gguf(tmp_path, gpu_backend, oracle):
    from test_gguf_moe import write_layer
    from test_gpu_moe import reference_ffn
    from gpu.gguf_moe import moe_layer
    E, H, I = 8, 2048, 2048
    arrays = write_layer(tmp_path / 'layer.gguf', 5, dims=(E, H, I), seed=9)
    moe = moe_layer(gpu_backend, tmp_path / 'layer.gguf', 5)
    try:
        assert (moe.top_k, moe.scale) == (2, 2.5)
        x = np.random.default_rng(10).normal(size=(6, H)).astype(np.float32)
        y, ids, _ = moe.forward(x)
        layer = {'router': arrays['router'], 'bias': arrays['bias'], 'gate': arrays['gate'].reshape(-1),
                 'up': arrays['up'].reshape(-1), 'down': arrays['down'].reshape(-1),
                 'shared': (arrays['shared_gate'].reshape(-1), arrays['shared_up'].reshape(-1),
                            arrays['shared_down'].reshape(-1))}
        want, want_ids = reference_ffn(oracle, layer, x, E, H, I, 2, 2.5)
        assert ids.tolist() == want_ids.tolist()
        assert np.linalg.norm(y - want) / np.linalg.norm(want) <= RTOL
    finally:
        moe.close()
