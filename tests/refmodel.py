"""Test infrastructure: the installed reference (baseline/_ref) driving this
library, and a small mixed-format packed checkpoint for it.

The reference's `kernels` package has the same name as this repository's
(glm-vx_b200/kernels), so it is loaded here under the alias `ref_kernels`;
`glm_vx` (the reference model code) has no clash and is imported as itself.
Nothing here is product code: the product is the library the reference's
unmodified classes call.
"""
import importlib
import sys
import types
from pathlib import Path

import numpy as np

from kernels.packed import LAYOUTS

ROOT = Path(__file__).resolve().parents[1]
REF = ROOT / 'baseline' / '_ref'


def available():
    return (REF / 'glm_vx' / 'model.py').exists() and (REF / 'kernels' / 'backend.py').exists()


def ref_kernels():
    """The reference's kernels package (backend.py, packed.py), aliased."""
    if 'ref_kernels' in sys.modules:
        return sys.modules['ref_kernels']
    mod = types.ModuleType('ref_kernels')  # the reference ships kernels/ as a namespace package
    mod.__path__ = [str(REF / 'kernels')]
    sys.modules['ref_kernels'] = mod
    importlib.import_module('ref_kernels.backend')
    importlib.import_module('ref_kernels.packed')
    return mod


def ref_glm_vx():
    if str(REF) not in sys.path:
        sys.path.append(str(REF))  # after this repository's packages
    import glm_vx.model
    import glm_vx.prefill  # noqa: F401
    return sys.modules['glm_vx']


def ref_vx_backend(library):
    """The reference's own VxBackend (kernels/backend.py) over `library`."""
    return ref_kernels().backend.VxBackend(str(library))


def dropin_config(layers=4, width=256):
    """The reference's tiny GLM-MoE-DSA config (glm_vx/tiny.py) widened so
    every projection is block-aligned for the packed formats: hidden and
    intermediate sizes `width` (256: IQ1_S / Q4_K rows; 2048: the tensor-core
    widths the expert-parallel layer needs), 8 routed experts + 1 shared,
    top-2, first layer dense, the last layer sharing the previous indexer
    selection."""
    from glm_vx.tiny import tiny_config
    c = tiny_config()
    c.update(hidden_size=width, vocab_size=512, num_hidden_layers=layers, num_attention_heads=4,
             num_key_value_heads=4, q_lora_rank=64, kv_lora_rank=32, qk_nope_head_dim=16, qk_rope_head_dim=8,
             qk_head_dim=24, v_head_dim=16, intermediate_size=width, moe_intermediate_size=width, n_routed_experts=8,
             num_experts_per_tok=2, index_head_dim=16, index_n_heads=4, index_topk=4,
             mlp_layer_types=['dense'] + ['sparse'] * (layers - 1),
             indexer_types=['full'] * (layers - 1) + ['shared'])
    return c


# Format of each projection (GGML kind): experts and dense MLPs IQ1_S,
# attention projections Q4_K / Q8_0, lm_head Q8_0, router and the narrow
# indexer head weights F32 (kind 0) -- every path of the packed contract.
def _kind_for(name, cols):
    if name == 'lm_head':
        return 8
    if '.mlp.gate' == name[-9:] or name.endswith('weights_proj'):
        return 0
    if '.mlp.' in name:
        return 19 if cols % 256 == 0 else 8
    if name.endswith(('q_a_proj', 'kv_a_proj_with_mqa', 'indexer.wk')) and cols % 256 == 0:
        return 12
    return 8 if cols % 32 == 0 else 0


def _random_blocks(rng, kind, rows, cols):
    """Random GGML blocks whose decoded weights have a std of about 1/sqrt(cols)."""
    block, size, _ = LAYOUTS[kind]
    nb = rows * cols // block
    raw = rng.integers(0, 256, size=(nb, size), dtype=np.uint8)
    unit = 1.0 / np.sqrt(cols)
    if kind == 8:    # d * int8, |q| ~ 73
        d = np.abs(rng.normal(size=nb)) * unit / 73
        raw[:, :2] = d.astype(np.float16).reshape(-1, 1).view(np.uint8)
    elif kind == 12:  # d * sc * q - dmin * m
        dd = (np.abs(rng.normal(size=(nb, 2))) * unit / 140).astype(np.float16)
        raw[:, :4] = dd.view(np.uint8)
    elif kind == 19:  # d * (2s + 1) * (grid +- 1/8)
        d = np.abs(rng.normal(size=nb)) * unit / 6.4
        raw[:, :2] = d.astype(np.float16).reshape(-1, 1).view(np.uint8)
    return raw.reshape(-1)


class PackedCheckpoint:
    """What glm_vx.model expects of a packed checkpoint (`linear`,
    `linear_batch`, name lookup), over host arrays: 2-D projections as raw
    GGML blocks, norms / biases / kv_b_proj / the embedding as f32."""

    def __init__(self, config, seed=0):
        ref_glm_vx()
        from glm_vx.model import GlmMoeDsaModel
        m = GlmMoeDsaModel(config, {}, None)
        c = m.config
        rng = np.random.default_rng(seed)
        self.packed, self.dense = {}, {}

        def proj(name, rows, cols):
            kind = _kind_for(name, cols)
            if kind == 0:
                w = (rng.normal(size=(rows, cols)) / np.sqrt(cols)).astype(np.float32)
                self.packed[name + '.weight'] = (w.reshape(-1).view(np.uint8), 0, (rows, cols))
            else:
                self.packed[name + '.weight'] = (_random_blocks(rng, kind, rows, cols), kind, (rows, cols))

        def norm(name, width, bias=False):
            self.dense[name + '.weight'] = (1.0 + 0.1 * rng.normal(size=width)).astype(np.float32)
            if bias:
                self.dense[name + '.bias'] = (0.1 * rng.normal(size=width)).astype(np.float32)

        H = m.hidden
        self.dense['model.embed_tokens.weight'] = rng.normal(size=(c['vocab_size'], H)).astype(np.float32)
        proj('lm_head', c['vocab_size'], H)
        norm('model.norm', H)
        for layer in range(m.n_layers):
            p = f'model.layers.{layer}'
            norm(p + '.input_layernorm', H)
            norm(p + '.post_attention_layernorm', H)
            a = p + '.self_attn'
            proj(a + '.q_a_proj', c['q_lora_rank'], H)
            norm(a + '.q_a_layernorm', c['q_lora_rank'])
            proj(a + '.q_b_proj', m.heads * (m.nope + m.rot), c['q_lora_rank'])
            proj(a + '.kv_a_proj_with_mqa', m.rank + m.rot, H)
            norm(a + '.kv_a_layernorm', m.rank)
            self.dense[a + '.kv_b_proj.weight'] = (rng.normal(size=(m.heads * (m.nope + m.value_dim), m.rank))
                                                   / np.sqrt(m.rank)).astype(np.float32)
            proj(a + '.o_proj', H, m.heads * m.value_dim)
            if m.indexer_types[layer] == 'full':
                proj(a + '.indexer.wq_b', m.index_heads * m.index_dim, c['q_lora_rank'])
                proj(a + '.indexer.wk', m.index_dim, H)
                norm(a + '.indexer.k_norm', m.index_dim, bias=True)
                proj(a + '.indexer.weights_proj', m.index_heads, H)
            mlp = p + '.mlp'
            if m.mlp_types[layer] == 'dense':
                for n, (r, k) in (('gate_proj', (c['intermediate_size'], H)), ('up_proj', (c['intermediate_size'], H)),
                                  ('down_proj', (H, c['intermediate_size']))):
                    proj(f'{mlp}.{n}', r, k)
            else:
                E, inter = int(c['n_routed_experts']), int(c['moe_intermediate_size'])
                proj(mlp + '.gate', E, H)
                self.dense[mlp + '.gate.e_score_correction_bias'] = (0.01 * rng.normal(size=E)).astype(np.float32)
                for e in ['shared_experts'] + [f'experts.{i}' for i in range(E)]:
                    for n, (r, k) in (('gate_proj', (inter, H)), ('up_proj', (inter, H)), ('down_proj', (H, inter))):
                        proj(f'{mlp}.{e}.{n}', r, k)

    def linear(self, name, x, backend):
        raw, kind, shape = self.packed[name]
        return backend.packed_matvec(raw, kind, shape, x)

    def linear_batch(self, name, x, backend):
        raw, kind, shape = self.packed[name]
        return backend.packed_linear_batch(raw, kind, shape, x)

    def __call__(self, name):
        if name in self.dense:
            return self.dense[name]
        raise KeyError(name)

    def packed_tensor(self, name):
        """(raw bytes, kind, shape) of a projection (gpu.decoder source protocol)."""
        return self.packed[name]

    def dense_tensor(self, name):
        """float32 array of a norm, bias, kv_b or the F32 embedding."""
        return self.dense[name]

    def kinds(self):
        return sorted({k for _, k, _ in self.packed.values()})


def greedy(model, prompt, new_tokens, grouped_prefill=True):
    """Greedy decode as the reference's generate loop does it
    (glm_vx/generate.py:86-109: prefill the prompt, argmax, feed back):
    returns (tokens, [logits of every sampled step])."""
    cache = model.new_cache()
    if grouped_prefill:
        logits = model.prefill_chunk(list(prompt), cache)  # glm_vx/prefill.py: batched projections
    else:
        for t in prompt[:-1]:
            model.prefill_token(int(t), cache)
        logits = model.forward(int(prompt[-1]), cache)
    tokens, all_logits = [], []
    for i in range(new_tokens):
        if not np.isfinite(logits).all():
            raise ValueError('nonfinite logits')
        all_logits.append(np.array(logits, copy=True))
        token = int(np.argmax(logits))
        tokens.append(token)
        if i + 1 < new_tokens:
            logits = model.forward(token, cache)
    return tokens, all_logits
