"""Sparse feed-forward layers straight from a GGUF checkpoint into HBM.

The reference borrows packed GGUF bytes one matrix at a time
(`GGUFStore.packed_rows`, glm_vx/gguf_reader.py:118-131) and hands them to the
backend per call (`GGUFCheckpoint.linear`, glm_vx/gguf_checkpoint.py:122-138).
Here a whole MoE layer's tensors -- router, correction bias, the stacked
gate/up/down expert arrays and the shared expert -- are read from the
memory-mapped file and uploaded once into an `MoELayer` (or, with
`experts=(first, count)`, this rank's slice into an `ExpertParallelMoE`), so
the experts stay resident and each step is a single layer call.

Tensor names are the llama.cpp GLM-DSA names the reference resolves
(glm_vx/gguf_checkpoint.py:29-30 for the router and bias, :84-88 for the
routed `ffn_{gate,up,down}_exps` stacks and the `_shexp` shared expert).
GGUF stores dimensions innermost first; shapes here are outermost first as
in the reference (`GGUFStore.shape`, glm_vx/gguf_reader.py:97).
"""
import numpy as np

NAMES = {'router': 'ffn_gate_inp.weight', 'bias': 'exp_probs_b.bias', 'gate': 'ffn_gate_exps.weight',
         'up': 'ffn_up_exps.weight', 'down': 'ffn_down_exps.weight', 'shared_gate': 'ffn_gate_shexp.weight',
         'shared_up': 'ffn_up_shexp.weight', 'shared_down': 'ffn_down_shexp.weight'}
F32 = 0


def open_reader(path_or_reader):
    """A gguf-py GGUFReader for a single-file checkpoint (or the reader itself)."""
    if hasattr(path_or_reader, 'tensors'):
        return path_or_reader
    import gguf
    return gguf.GGUFReader(path_or_reader)


def _field(reader, key, default=None):
    field = reader.fields.get(key)
    return default if field is None else field.contents()


def layer_tensors(reader, layer):
    """{piece: (array, kind, shape)} of one sparse layer; packed pieces are the
    file's bytes (uint8, no copy), router and bias f32.  Raises KeyError for a
    missing routed piece; shared pieces are optional together."""
    tensors = {t.name: t for t in reader.tensors}
    out = {}
    for piece, suffix in NAMES.items():
        name = f'blk.{layer}.{suffix}'
        t = tensors.get(name)
        if t is None:
            if piece.startswith('shared'):
                continue
            raise KeyError(name)
        shape = tuple(int(n) for n in reversed(t.shape))
        kind = int(t.tensor_type)
        data = np.asarray(t.data)
        if piece in ('router', 'bias'):
            if kind != F32:
                raise ValueError(f'{name} must be F32')
            arr = data.reshape(shape).astype(np.float32, copy=False)
        else:
            arr = data.reshape(-1).view(np.uint8)
        out[piece] = (arr, kind, shape)
    shared = [p for p in ('shared_gate', 'shared_up', 'shared_down') if p in out]
    if shared and len(shared) != 3:
        raise KeyError(f'blk.{layer}: shared expert needs gate, up and down')
    return out


def _check(t):
    kinds = {t[p][1] for p in ('gate', 'up', 'down')}
    if len(kinds) != 1:
        raise ValueError('gate, up and down experts must share one format')
    E, inter, hidden = t['gate'][2]
    if t['up'][2] != (E, inter, hidden) or t['down'][2] != (E, hidden, inter):
        raise ValueError('expert stacks must be [E, inter, hidden] (gate, up) and [E, hidden, inter] (down)')
    if t['router'][2] != (E, hidden) or t['bias'][2] != (E,):
        raise ValueError('router must be [E, hidden] and bias [E]')
    return kinds.pop(), E, hidden, inter


def moe_layer(backend, source, layer, *, top_k=None, scale=None):
    """MoELayer (gpu/moe.py) of GGUF block `layer`, experts resident on the
    backend's device.  top_k and the routed scale default to the file's
    glm-dsa.expert_used_count / glm-dsa.expert_weights_scale."""
    from .moe import MoELayer
    reader = open_reader(source)
    t = layer_tensors(reader, layer)
    kind, E, hidden, inter = _check(t)
    top_k = int(top_k if top_k is not None else _field(reader, 'glm-dsa.expert_used_count'))
    scale = float(scale if scale is not None else _field(reader, 'glm-dsa.expert_weights_scale'))
    shared = tuple(t[p][0] for p in ('shared_gate', 'shared_up', 'shared_down')) if 'shared_gate' in t else None
    return MoELayer(backend, t['router'][0], t['bias'][0], kind, t['gate'][0], t['up'][0], t['down'][0], hidden,
                    inter, top_k, scale, shared=shared)


def expert_slice(array, experts_total, first, count):
    """Bytes of experts [first, first + count) of a packed [E, ...] stack."""
    per = array.nbytes // experts_total
    if per * experts_total != array.nbytes or not 0 <= first <= first + count <= experts_total:
        raise ValueError('expert slice outside the stack')
    return array[first * per:(first + count) * per]


def expert_parallel_layer(source, layer, rank, world, backend, *, top_k=None, scale=None, max_tokens=32):
    """ExpertParallelLayer (gpu/ep.py) holding this rank's experts
    [rank*E/world, (rank+1)*E/world) of GGUF block `layer` on `backend`'s
    device; router, bias and shared expert replicated.  Connect it to the
    other ranks (connect_ipc) before its first step."""
    from .ep import ExpertParallelLayer, experts_per_rank
    reader = open_reader(source)
    t = layer_tensors(reader, layer)
    kind, E, hidden, inter = _check(t)
    per = experts_per_rank(E, world)
    top_k = int(top_k if top_k is not None else _field(reader, 'glm-dsa.expert_used_count'))
    scale = float(scale if scale is not None else _field(reader, 'glm-dsa.expert_weights_scale'))
    part = {p: expert_slice(t[p][0], E, rank * per, per) for p in ('gate', 'up', 'down')}
    shared = tuple(t[p][0] for p in ('shared_gate', 'shared_up', 'shared_down')) if 'shared_gate' in t else None
    return ExpertParallelLayer(backend, rank, world, t['router'][0], t['bias'][0], kind, part['gate'], part['up'],
                               part['down'], E, hidden, inter, top_k, scale, shared=shared, max_tokens=max_tokens)
