"""GGUF -> resident MoE layer mapping (gpu/gguf_moe.py): tensor names,
shapes, kinds and bytes of a sparse layer read back from a GGUF file written
with gguf-py, expert slices for expert parallelism, and the errors for
missing or inconsistent tensors.  No GPU: only the host mapping."""
import numpy as np
import pytest

gguf = pytest.importorskip('gguf')

E, H, I, K = 4, 512, 256, 2


def write_layer(path, layer, *, shared=True, seed=0, kind=19, drop=None, dims=(E, H, I)):
    """A glm-dsa GGUF holding one sparse layer at block `layer`; returns the arrays written."""
    from kernels.packed import LAYOUTS
    E, H, I = dims
    block, size, _ = LAYOUTS[kind]
    rng = np.random.default_rng(seed)

    def packed(e, rows, cols):
        raw = rng.integers(0, 256, size=(e, rows, cols // block, size), dtype=np.uint8)
        raw[..., :2] = (np.abs(rng.normal(size=raw.shape[:3] + (1,))) * 0.02).astype(np.float16).view(np.uint8)
        return raw.reshape(e, rows, cols // block * size)

    arrays = {'router': (rng.normal(size=(E, H)) * 0.02).astype(np.float32),
              'bias': (rng.normal(size=E) * 0.01).astype(np.float32),
              'gate': packed(E, I, H), 'up': packed(E, I, H), 'down': packed(E, H, I)}
    if shared:
        arrays.update(shared_gate=packed(1, I, H)[0], shared_up=packed(1, I, H)[0], shared_down=packed(1, H, I)[0])
    from gpu.gguf_moe import NAMES
    w = gguf.GGUFWriter(str(path), 'glm-dsa')
    w.add_uint32('glm-dsa.expert_used_count', K)
    w.add_float32('glm-dsa.expert_weights_scale', 2.5)
    for piece, arr in arrays.items():
        if piece == drop:
            continue
        name = f'blk.{layer}.{NAMES[piece]}'
        if arr.dtype == np.float32:
            w.add_tensor(name, arr)
        else:
            w.add_tensor(name, arr, raw_dtype=gguf.GGMLQuantizationType(kind))
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    return arrays


def test_layer_tensors_read_back(tmp_path):
    from gpu.gguf_moe import layer_tensors, open_reader
    arrays = write_layer(tmp_path / 'm.gguf', 3)
    t = layer_tensors(open_reader(tmp_path / 'm.gguf'), 3)
    assert t['gate'][2] == (E, I, H) and t['up'][2] == (E, I, H) and t['down'][2] == (E, H, I)
    assert t['router'][2] == (E, H) and t['bias'][2] == (E,)
    assert t['shared_gate'][2] == (I, H) and t['shared_down'][2] == (H, I)
    for piece, arr in arrays.items():
        got = t[piece][0]
        if arr.dtype == np.float32:
            assert got.dtype == np.float32 and np.array_equal(got, arr)
        else:
            assert t[piece][1] == 19
            assert got.dtype == np.uint8 and got.tobytes() == arr.tobytes()


def test_expert_slice_and_errors(tmp_path):
    from gpu.gguf_moe import expert_slice, layer_tensors, open_reader, _check
    arrays = write_layer(tmp_path / 'm.gguf', 0, shared=False)
    t = layer_tensors(open_reader(tmp_path / 'm.gguf'), 0)
    assert 'shared_gate' not in t
    assert _check(t) == (19, E, H, I)
    part = expert_slice(t['down'][0], E, 1, 2)
    assert part.tobytes() == arrays['down'][1:3].tobytes()
    with pytest.raises(ValueError, match='outside'):
        expert_slice(t['down'][0], E, 3, 2)
    with pytest.raises(KeyError):
        layer_tensors(open_reader(tmp_path / 'm.gguf'), 1)
    write_layer(tmp_path / 'd.gguf', 0, drop='up')
    with pytest.raises(KeyError, match='ffn_up_exps'):
        layer_tensors(open_reader(tmp_path / 'd.gguf'), 0)
    write_layer(tmp_path / 's.gguf', 0, drop='shared_up')
    with pytest.raises(KeyError, match='shared expert'):
        layer_tensors(open_reader(tmp_path / 's.gguf'), 0)
