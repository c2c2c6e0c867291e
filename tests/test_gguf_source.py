"""GGUF checkpoint source (gpu/gguf_source.py) on the CPU: split-file
validation as the reference's GGUFStore does it (glm_vx/gguf_reader.py:25-63),
the model-name mapping (glm_vx/gguf_checkpoint.py:85-101) and byte identity of
what the decoder uploads, against a synthetic GLM-DSA checkpoint written with
gguf-py (tests/gguf_fixture.py); and the reference's own GGUFCheckpoint
accepting that file, so the fixture is a faithful GLM-DSA GGUF."""
import shutil

import numpy as np
import pytest

import refmodel

pytestmark = pytest.mark.skipif(not refmodel.available(), reason='reference not installed in baseline/_ref')


@pytest.fixture(scope='module')
def written(tmp_path_factory):
    import gguf_fixture
    refmodel.ref_glm_vx()
    config = refmodel.dropin_config(layers=3, width=256)
    ckpt = refmodel.PackedCheckpoint(config, seed=3)
    d = tmp_path_factory.mktemp('gguf')
    (d / 'split').mkdir()
    (d / 'single').mkdir()
    split = gguf_fixture.write_checkpoint(ckpt, config, d / 'split' / 'tiny.gguf', split_max_tensors=20)
    single = gguf_fixture.write_checkpoint(ckpt, config, d / 'single' / 'tiny.gguf')
    return config, ckpt, split, single


def test_split_and_single_file_give_the_same_bytes(written):
    from gpu.gguf_source import GGUFSource
    config, ckpt, split, single = written
    assert len(split) > 2 and all(p.name.endswith(f'-of-{len(split):05}.gguf') for p in split)
    for path in (split[1], single[0], split[0].parent):
        src = GGUFSource(path, config)
        try:
            for name, (raw, kind, shape) in ckpt.packed.items():
                got, gkind, gshape = src.packed_tensor(name)
                assert (gkind, tuple(gshape)) == (kind, tuple(shape)), name
                assert got.tobytes() == np.ascontiguousarray(raw).view(np.uint8).tobytes(), name
            for name, want in ckpt.dense.items():
                assert np.array_equal(src.dense_tensor(name), want), name
        finally:
            src.close()


def test_split_validation(written, tmp_path):
    from gpu.gguf_source import GGUFError, GGUFSource
    config, _, split, _ = written
    d = tmp_path / 'broken'
    d.mkdir()
    for p in split[:-1]:  # the last file missing
        shutil.copy(p, d / p.name)
    with pytest.raises(GGUFError, match='missing GGUF split file'):
        GGUFSource(d / split[0].name)
    shutil.copy(split[-1], d / split[-1].name)
    GGUFSource(d / split[0].name).close()
    # a shard renamed out of order: its split.no no longer matches
    (d / split[0].name).rename(d / 'x.gguf')
    (d / split[1].name).rename(d / split[0].name)
    (d / 'x.gguf').rename(d / split[1].name)
    with pytest.raises(GGUFError, match='split index/count'):
        GGUFSource(d / split[0].name)


def test_config_mismatch_and_unknown_names(written):
    from gpu.gguf_source import GGUFError, GGUFSource
    config, _, _, single = written
    bad = dict(config, hidden_size=512)
    with pytest.raises(GGUFError, match='embedding_length'):
        GGUFSource(single[0], bad)
    src = GGUFSource(single[0], config)
    try:
        with pytest.raises(KeyError):
            src.packed_tensor('model.layers.0.self_attn.nonexistent.weight')
        with pytest.raises(KeyError):
            src.packed_tensor(f'model.layers.1.mlp.experts.{config["n_routed_experts"]}.gate_proj.weight')
    finally:
        src.close()


def test_reference_loader_accepts_the_fixture(written):
    """The reference's GGUFCheckpoint validates the metadata and manifest and
    rebuilds kv_b from attn_k_b / attn_v_b to the checkpoint's values."""
    refmodel.ref_glm_vx()
    from glm_vx.gguf_checkpoint import GGUFCheckpoint
    config, ckpt, split, _ = written
    ref = GGUFCheckpoint(str(split[0]), config)
    try:
        name = 'model.layers.0.self_attn.kv_b_proj.weight'
        assert np.allclose(ref.tensor(name), ckpt.dense[name], rtol=0, atol=0)
    finally:
        ref.close()
