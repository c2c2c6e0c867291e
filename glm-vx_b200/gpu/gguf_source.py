"""A GLM-DSA GGUF checkpoint (one file or a split set) as the weight source of
the resident decoder (gpu/decoder.py) and of the expert-parallel layers.

The reference reads split GGUF files through `GGUFStore`
(glm_vx/gguf_reader.py:17-91: split naming `<stem>-0000i-of-0000n.gguf`, the
`split.no` / `split.count` / `split.tensors.count` manifest, tensor spans
inside their file, no duplicates, little-endian only) and maps model names to
llama.cpp's GLM-DSA names in `GGUFCheckpoint._resolve`
(glm_vx/gguf_checkpoint.py:15-31, 85-101: `blk.<i>.<piece>`, experts stacked
by expert id in `ffn_<part>_exps`, kv_b rebuilt from `attn_k_b` transposed
per head and `attn_v_b`).  It decodes weights on the host per call.  Here the
file is memory-mapped once and the decoder copies each tensor's packed bytes
straight to HBM: projections stay in their GGUF format (the kernels decode
them), an expert-parallel rank takes only its own experts' slices of the
stacked arrays (no other rank's bytes are read), and the few dense tensors
that are stored quantized (kv_b halves, an embedding) are decoded on the
device by the library's unpack kernel.

Interface used by ResidentDecoder: packed_tensor(name) -> (uint8 bytes, GGML
kind, (rows, cols)) for a projection or one expert; dense_tensor(name) ->
float32 array for norms, biases, kv_b and an F32 embedding.  Model names are
the Hugging Face ones the reference model uses.
"""
import math
import re
from pathlib import Path

import numpy as np

F32, F16 = 0, 1

# Hugging Face name suffix -> llama.cpp GLM-DSA tensor (the GGUF format's
# names, as the reference's conversion inverse lists them).
_LAYER_NAMES = {
    'input_layernorm.weight': 'attn_norm.weight',
    'post_attention_layernorm.weight': 'ffn_norm.weight',
    'self_attn.q_a_proj.weight': 'attn_q_a.weight',
    'self_attn.q_a_layernorm.weight': 'attn_q_a_norm.weight',
    'self_attn.q_b_proj.weight': 'attn_q_b.weight',
    'self_attn.kv_a_proj_with_mqa.weight': 'attn_kv_a_mqa.weight',
    'self_attn.kv_a_layernorm.weight': 'attn_kv_a_norm.weight',
    'self_attn.o_proj.weight': 'attn_output.weight',
    'self_attn.indexer.wq_b.weight': 'indexer.attn_q_b.weight',
    'self_attn.indexer.wk.weight': 'indexer.attn_k.weight',
    'self_attn.indexer.k_norm.weight': 'indexer.k_norm.weight',
    'self_attn.indexer.k_norm.bias': 'indexer.k_norm.bias',
    'self_attn.indexer.weights_proj.weight': 'indexer.proj.weight',
    'mlp.gate.weight': 'ffn_gate_inp.weight',
    'mlp.gate.e_score_correction_bias': 'exp_probs_b.bias',
}
_GLOBAL_NAMES = {'model.embed_tokens.weight': 'token_embd.weight', 'model.norm.weight': 'output_norm.weight',
                 'lm_head.weight': 'output.weight'}
_SPLIT = re.compile(r'(.*)-(\d{5})-of-(\d{5})\.gguf')


class GGUFError(ValueError):
    pass


def split_paths(path):
    """The files of a checkpoint: a directory holding one checkpoint, a
    single file, or the first (any) file of a `-0000i-of-0000n` split set."""
    path = Path(path)
    if path.is_dir():
        first = sorted(path.glob('*-00001-of-*.gguf')) or sorted(path.glob('*.gguf'))
        if len(first) != 1:
            raise GGUFError('directory must hold exactly one GGUF checkpoint')
        path = first[0]
    m = _SPLIT.fullmatch(path.name)
    if not m:
        return [path]
    count = int(m[3])
    if not 1 <= count <= 1024 or not 1 <= int(m[2]) <= count:
        raise GGUFError('invalid split index/count in ' + path.name)
    return [path.with_name(f'{m[1]}-{i:05}-of-{count:05}.gguf') for i in range(1, count + 1)]


class GGUFSource:
    """Memory-mapped GLM-DSA GGUF checkpoint (see the module docstring).
    `config` (the model config dict) is checked against the file's metadata;
    `backend` (a GPUBackend) decodes quantized dense tensors on the device."""

    def __init__(self, path, config=None, backend=None):
        import gguf
        self.backend = backend
        self.paths = split_paths(path)
        self.readers, self.tensors, self.metadata = [], {}, {}
        total = None
        for index, p in enumerate(self.paths):
            if not p.exists():
                raise GGUFError(f'missing GGUF split file {p.name}')
            reader = gguf.GGUFReader(p)
            if reader.endianess != gguf.GGUFEndian.LITTLE:
                raise GGUFError('only little-endian GGUF is supported')
            self.readers.append(reader)
            fields = {k: v.contents() for k, v in reader.fields.items() if not k.startswith('GGUF.')}
            if index == 0:
                self.metadata = fields
            if len(self.paths) > 1:
                if fields.get('split.no') != index or fields.get('split.count') != len(self.paths):
                    raise GGUFError(f'{p.name}: split index/count do not match its file name')
                n = fields.get('split.tensors.count')
                if type(n) is not int or n < 1 or (total is not None and n != total):
                    raise GGUFError(f'{p.name}: missing or inconsistent split tensor count')
                total = n
            elif fields.get('split.count', 1) != 1:
                raise GGUFError('a split GGUF checkpoint is missing its other files')
            for key, value in fields.items():  # later shards may omit model metadata, not contradict it
                if key.startswith(('general.architecture', 'glm-dsa.')) and self.metadata.get(key, value) != value:
                    raise GGUFError('inconsistent GGUF metadata: ' + key)
            size, spans = p.stat().st_size, []
            for t in reader.tensors:
                shape = tuple(int(n) for n in reversed(t.shape))
                block, block_bytes = gguf.GGML_QUANT_SIZES[t.tensor_type]
                if not shape or min(shape) <= 0 or shape[-1] % block:
                    raise GGUFError('invalid tensor shape: ' + t.name)
                nbytes = math.prod(shape) // block * block_bytes
                if t.n_bytes != nbytes or t.data_offset < reader.data_offset or t.data_offset + nbytes > size:
                    raise GGUFError('tensor outside its file: ' + t.name)
                if t.name in self.tensors:
                    raise GGUFError('duplicate tensor: ' + t.name)
                spans.append((t.data_offset, t.data_offset + nbytes))
                self.tensors[t.name] = t
            spans.sort()
            if any(a[1] > b[0] for a, b in zip(spans, spans[1:])):
                raise GGUFError('overlapping tensor storage')
        if total is not None and total != len(self.tensors):
            raise GGUFError(f'split manifest lists {total} tensors, the files hold {len(self.tensors)}')
        if self.metadata.get('general.architecture') != 'glm-dsa':
            raise GGUFError('GGUF architecture must be glm-dsa')
        if config is not None:
            self.check_config(config)

    # -------------------------------------------------------------- metadata
    def check_config(self, c):
        """The dimensions the decoder sizes its buffers from must be the file's."""
        m = lambda k: self.metadata.get('glm-dsa.' + k)
        checks = {'embedding_length': c['hidden_size'], 'vocab_size': c['vocab_size'],
                  'attention.head_count': c['num_attention_heads'], 'attention.q_lora_rank': c['q_lora_rank'],
                  'attention.kv_lora_rank': c['kv_lora_rank'], 'rope.dimension_count': c['qk_rope_head_dim'],
                  'attention.key_length_mla': c['qk_nope_head_dim'] + c['qk_rope_head_dim'],
                  'attention.value_length_mla': c['v_head_dim'], 'expert_count': c['n_routed_experts'],
                  'expert_used_count': c['num_experts_per_tok'],
                  'expert_feed_forward_length': c['moe_intermediate_size'],
                  'feed_forward_length': c['intermediate_size'],
                  'leading_dense_block_count': c['first_k_dense_replace']}
        for key, want in checks.items():
            if m(key) != want:
                raise GGUFError(f'GGUF/config mismatch: glm-dsa.{key} = {m(key)}, config {want}')
        mtp = m('nextn_predict_layers') or 0
        if m('block_count') != c['num_hidden_layers'] + mtp:
            raise GGUFError('GGUF block count does not match the decoder layers plus the MTP layers')

    # ----------------------------------------------------------------- names
    def resolve(self, name):
        """Model tensor name -> (GGUF tensor name, expert index or None)."""
        if name in _GLOBAL_NAMES:
            return _GLOBAL_NAMES[name], None
        m = re.fullmatch(r'model\.layers\.(\d+)\.(.+)', name)
        if not m:
            raise KeyError(name)
        prefix, suffix = f'blk.{int(m[1])}.', m[2]
        if suffix == 'self_attn.kv_b_proj.weight':
            return prefix + 'attn_kv_b', None  # rebuilt from attn_k_b and attn_v_b
        if suffix in _LAYER_NAMES:
            return prefix + _LAYER_NAMES[suffix], None
        e = re.fullmatch(r'mlp\.experts\.(\d+)\.(gate|up|down)_proj\.weight', suffix)
        if e:
            return prefix + f'ffn_{e[2]}_exps.weight', int(e[1])
        s = re.fullmatch(r'mlp\.(shared_experts\.)?(gate|up|down)_proj\.weight', suffix)
        if s:
            return prefix + f'ffn_{s[2]}' + ('_shexp' if s[1] else '') + '.weight', None
        raise KeyError(name)

    def _tensor(self, gname):
        t = self.tensors.get(gname)
        if t is None:
            raise KeyError(gname)
        return t, tuple(int(n) for n in reversed(t.shape))

    # ----------------------------------------------------------- the tensors
    def packed_tensor(self, name):
        """(uint8 view of the file's bytes, GGML kind, (rows, cols)) of a
        projection, or of one expert of a stacked expert array."""
        gname, expert = self.resolve(name)
        t, shape = self._tensor(gname)
        data = np.asarray(t.data)
        if expert is not None:
            if len(shape) != 3 or not 0 <= expert < shape[0]:
                raise KeyError(f'{name}: no expert {expert} in {gname} {shape}')
            data, shape = data[expert], shape[1:]
        if len(shape) != 2:
            raise KeyError(f'{name}: {gname} is not a matrix {shape}')
        raw = data.view(np.uint8).reshape(-1)
        return raw, int(t.tensor_type), shape

    def dense_tensor(self, name):
        """float32 array of a norm, bias, embedding or the rebuilt kv_b."""
        gname, expert = self.resolve(name)
        if gname.endswith('attn_kv_b'):
            k = self._decoded(gname[:-len('attn_kv_b')] + 'attn_k_b.weight')  # [heads][rank][nope]
            v = self._decoded(gname[:-len('attn_kv_b')] + 'attn_v_b.weight')  # [heads][v][rank]
            if k.ndim != 3 or v.ndim != 3 or k.shape[0] != v.shape[0] or k.shape[1] != v.shape[2]:
                raise GGUFError(f'attn_k_b {k.shape} / attn_v_b {v.shape} do not form kv_b')
            return np.concatenate((k.transpose(0, 2, 1), v), axis=1).reshape(-1, k.shape[1])
        if expert is not None:
            raise KeyError(name)
        return self._decoded(gname)

    def _decoded(self, gname):
        t, shape = self._tensor(gname)
        kind = int(t.tensor_type)
        data = np.asarray(t.data)
        if kind == F32:
            return data.reshape(shape).astype(np.float32, copy=False)
        if kind == F16:
            return data.reshape(shape).astype(np.float32)
        if self.backend is None:
            raise GGUFError(f'{gname} is stored quantized (kind {kind}); pass a GPU backend to decode it')
        from kernels.packed import LAYOUTS
        block, _, _ = LAYOUTS[kind]
        count = math.prod(shape)
        out = self.backend.unpack(data.view(np.uint8).reshape(-1), kind, count // block)
        return np.asarray(out, np.float32).reshape(shape)

    def close(self):
        for r in self.readers:
            mm = getattr(r, 'data', None)
            if hasattr(mm, '_mmap'):
                mm._mmap.close()
        self.readers, self.tensors = [], {}
