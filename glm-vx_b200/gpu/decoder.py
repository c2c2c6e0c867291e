"""Resident batched greedy decode of a GLM-MoE-DSA model on the B200.

The reference decodes one token of one request per call, through host
round trips per kernel (glm_vx/model.py:359-392 `_forward`, greedy loop
glm_vx/generate.py:86-109, scheduler glm_vx/scheduler.py:160-166).  Here the
whole model is held in HBM and a decode step advances B sequences by one
token each, entirely on the device: embedding -> per layer (rmsnorm,
absorbed-MLA attention with the DSA indexer, residual, rmsnorm, dense MLP or
routed + shared MoE, residual) -> final norm -> lm_head -> argmax, whose ids
are the next step's embedding input.  A step is captured once as a CUDA
graph and replayed; the host only copies prompt tokens in and generated
tokens (and, on request, logits) out.

Per token the arithmetic follows the reference model exactly:
  attention (model.py:178-237): q_a -> rmsnorm(1e-6) -> q_b; kv_a ->
    rmsnorm(latent, 1e-6) + rope(rope key); the indexer (model.py:136-176:
    wq_b, wk -> layernorm(1e-6) -> rope of the first rot dims, head weights
    * index_heads^-0.5, scores, stable top-k over every cached position) on
    'full' layers, the previous layer's selection on 'shared' ones; latent
    queries kv_b[h,:nope]^T q_nope, rope queries, the absorbed attention
    over the selected latents, kv_b[h,nope:] . attended, o_proj;
  feed-forward (model.py:289-324): SwiGLU MLP, or router -> sigmoid top-k
    -> experts in ascending id + shared expert (csrc/moe.cu).
Every projection is a packed GGML matrix (or F32, GGUF kind 0) run by the
packed GEMM for the batch; kv_b stays F32 as the reference keeps it.

Weights come from a `source` with two methods: packed_tensor(name) ->
(raw uint8 bytes, kind, (rows, cols)) for projections, dense_tensor(name) ->
float32 array for norms, biases, kv_b and an F32 embedding; a Q8_0 embedding
is a packed tensor.  `SyntheticWeights` generates a config's random weights
on the device instead (counter-based, seeded), for configurations too large
to build on the host.
"""
import ctypes as C
import hashlib
import math

import numpy as np

from . import runtime as rt
from kernels.packed import LAYOUTS


def _layer_types(c, n_layers):
    """Per-layer indexer ('full'/'shared') and MLP ('dense'/'sparse') types,
    as the reference model derives them (model.py:83-97)."""
    types = c.get('indexer_types')
    if types is None:
        pattern = c.get('index_topk_pattern')
        if pattern is not None:
            types = [{'F': 'full', 'S': 'shared'}[x] for x in pattern] if isinstance(pattern, str) else list(pattern)
        else:
            freq = max(int(c.get('index_topk_freq', 1)), 1)
            offset = int(c.get('index_skip_topk_offset', 2))
            types = ['full' if max(i - offset + 1, 0) % freq == 0 else 'shared' for i in range(n_layers)]
    dense = min(int(c.get('first_k_dense_replace', 1)), n_layers)
    mlp = list(c.get('mlp_layer_types') or (['dense'] * dense + ['sparse'] * (n_layers - dense)))
    return list(types), mlp


def rope_tables(d, positions, theta):
    """cos/sin [positions][d/2] float32 with the reference's arithmetic
    (kernels/backend.py:32-39) at every position."""
    from kernels.backend import _rope_table
    cos = np.empty((positions, d // 2), np.float32)
    sin = np.empty((positions, d // 2), np.float32)
    for p in range(positions):
        cos[p], sin[p] = _rope_table(d, float(p), float(theta))
    return cos, sin


class SyntheticWeights:
    """Random-init weights of `config` generated on the device from `seed`
    (glmvx_fill_random: counter-based hash per element; packed blocks get
    random bytes with |N(0,1)| * scale fp16 block scales, F32 tensors N(0,1)
    * scale, norms 1).  Formats follow BASELINE config 4: IQ1_S experts and
    dense MLP, Q4_K attention projections, Q8_0 embedding and lm_head, F32
    routers, indexer head weights and kv_b."""

    def __init__(self, config, seed=0, attention_kind=None):
        """attention_kind: GGML kind of the attention projections (default
        Q4_K where the width allows, as config 4; 8 for config 3's Q8_0)."""
        self.config, self.seed, self.attention_kind = dict(config), int(seed), attention_kind

    def fill(self, lib, ptr, kind, count, scale, key, ones, stream):
        """Generate tensor `key` at device address ptr (its seed is a hash of
        the model seed and the tensor name, so every rank and every
        configuration derives the same bytes for the same tensor)."""
        digest = hashlib.sha256(f'{self.seed}:{key}'.encode()).digest()
        rt.check(lib, lib.glmvx_fill_random(ptr, kind, count, int.from_bytes(digest[:8], 'little'), scale,
                                            int(ones), stream), 'glmvx_fill_random')

    def kind(self, name, shape):
        if name in ('lm_head', 'model.embed_tokens'):
            return 8
        if name.endswith('.mlp.gate') or name.endswith('weights_proj') or name.endswith('kv_b_proj'):
            return 0
        if '.mlp.' in name:
            return 19
        if self.attention_kind is not None:
            return self.attention_kind
        return 12 if shape[1] % 256 == 0 else 8

    @staticmethod
    def scale(kind, cols):
        """Block-scale multiplier (packed: fp16 d = |N(0,1)| * scale, the
        BASELINE distributions: IQ1_S 0.02, Q4_K and Q8_0 0.01) or the F32
        standard deviation (1/sqrt(cols))."""
        return {19: 0.02, 12: 0.01, 8: 0.01}.get(kind, 1.0 / math.sqrt(cols))


class ResidentDecoder:
    """B sequences of one model decoding together on `backend`'s device.

    capacity: cache rows per sequence (prompt + generated tokens).
    moe_layer_factory (optional): callable(layer_index, loader) returning an
    object with forward_device(y, x, tokens, ids=None, weights=None) for the
    sparse layers (e.g. an expert-parallel layer); default: the whole layer
    on this GPU (glmvx_moe_ffn)."""

    def __init__(self, backend, config, source, batch, capacity, layers=None, moe_layer_factory=None):
        self.backend, self.lib = backend, backend.lib
        c = self.config = dict(config)
        self.n_layers = int(layers if layers is not None else c['num_hidden_layers'])
        self.B, self.capacity = int(batch), int(capacity)
        if not 1 <= self.B <= 64:
            raise ValueError('batch must be 1..64 sequences (packed GEMM batch)')
        self.hidden, self.heads = int(c['hidden_size']), int(c['num_attention_heads'])
        self.rank, self.nope, self.rot = int(c['kv_lora_rank']), int(c['qk_nope_head_dim']), int(c['qk_rope_head_dim'])
        self.vdim, self.q_lora = int(c['v_head_dim']), int(c['q_lora_rank'])
        self.ih, self.idim, self.topk = int(c['index_n_heads']), int(c['index_head_dim']), int(c['index_topk'])
        self.vocab, self.eps = int(c['vocab_size']), float(c.get('rms_norm_eps', 1e-5))
        self.k, self.scale_r = int(c.get('num_experts_per_tok', 8)), float(c.get('routed_scaling_factor', 1.0))
        rope = c.get('rope_parameters') or {'rope_theta': c.get('rope_theta', 10000)}
        self.theta = float(rope.get('rope_theta', c.get('rope_theta', 10000)))
        if c.get('attention_bias', False):
            raise ValueError('attention biases are not supported by the resident decoder')
        if c.get('tie_word_embeddings', False):
            raise ValueError('tied embeddings are not supported by the resident decoder')
        self.indexer_types, self.mlp_types = _layer_types(c, int(c['num_hidden_layers']))
        self.indexer_types, self.mlp_types = self.indexer_types[:self.n_layers], self.mlp_types[:self.n_layers]
        if self.indexer_types[0] != 'full':
            raise ValueError('the first layer must have a full indexer')
        self._bufs = []
        self._moe_factory = moe_layer_factory
        self._synthetic = isinstance(source, SyntheticWeights)
        self.source = source
        backend._begin()
        self.s = backend.stream.handle
        self._load()
        self._alloc_state()
        self._graph = None

    # ------------------------------------------------------------ memory
    def _dev(self, nbytes):
        buf = rt.DeviceBuffer(max(int(nbytes), 256))
        self._bufs.append(buf)
        return buf

    def _put(self, array):
        array = np.ascontiguousarray(array)
        buf = self._dev(array.nbytes)
        buf.upload(array, self.s)
        return buf.ptr

    def _fill(self, kind, nbytes, count, scale, key, ones=False):
        """Device buffer of synthetic weights for tensor `key` (see SyntheticWeights)."""
        buf = self._dev(nbytes)
        self.source.fill(self.lib, buf.ptr, kind, count, scale, key, ones, self.s)
        return buf.ptr

    def _proj(self, name, rows, cols):
        """(device pointer, kind, rows, cols) of projection `name`."""
        if self._synthetic:
            kind = self.source.kind(name, (rows, cols))
            block, size, _ = LAYOUTS[kind] if kind else (1, 4, 'f32')
            count = rows * cols // block
            return self._fill(kind, count * size, count, self.source.scale(kind, cols), name), kind, rows, cols
        raw, kind, shape = self.source.packed_tensor(name + '.weight')
        if tuple(shape) != (rows, cols):
            raise ValueError(f'{name}: shape {shape}, expected {(rows, cols)}')
        return self._put(np.ascontiguousarray(raw).view(np.uint8)), int(kind), rows, cols

    def _vec(self, name, n, ones=True):
        if self._synthetic:  # norms 1, biases N(0, 0.01)
            return self._fill(0, 4 * n, n, 0.01, name, ones=ones)
        a = np.asarray(self.source.dense_tensor(name), np.float32)
        if a.shape != (n,):
            raise ValueError(f'{name}: shape {a.shape}, expected ({n},)')
        return self._put(a)

    def _load(self):
        c, H = self.config, self.hidden
        self.layers = []
        if self._synthetic:
            self.embed = self._proj('model.embed_tokens', self.vocab, H)
        else:
            try:
                self.embed = self._proj('model.embed_tokens', self.vocab, H)
            except KeyError:
                e = np.asarray(self.source.dense_tensor('model.embed_tokens.weight'), np.float32)
                self.embed = (self._put(e), 0, self.vocab, H)
        self.lm_head = self._proj('lm_head', self.vocab, H)
        self.final_norm = self._vec('model.norm.weight', H)
        for i in range(self.n_layers):
            p, a = f'model.layers.{i}', f'model.layers.{i}.self_attn'
            L = {'in_norm': self._vec(p + '.input_layernorm.weight', H),
                 'post_norm': self._vec(p + '.post_attention_layernorm.weight', H),
                 'q_a': self._proj(a + '.q_a_proj', self.q_lora, H),
                 'q_a_norm': self._vec(a + '.q_a_layernorm.weight', self.q_lora),
                 'q_b': self._proj(a + '.q_b_proj', self.heads * (self.nope + self.rot), self.q_lora),
                 'kv_a': self._proj(a + '.kv_a_proj_with_mqa', self.rank + self.rot, H),
                 'kv_a_norm': self._vec(a + '.kv_a_layernorm.weight', self.rank),
                 'o': self._proj(a + '.o_proj', H, self.heads * self.vdim)}
            # kv_b [heads][nope + v][rank] f32, as the reference keeps it: the
            # query absorption reads its first nope rows of each head, the
            # value absorption the last v rows.
            if self._synthetic:
                n = self.heads * (self.nope + self.vdim) * self.rank
                kvb = self._fill(0, 4 * n, n, 1.0 / math.sqrt(self.rank), a + '.kv_b_proj')
            else:
                w = np.asarray(self.source.dense_tensor(a + '.kv_b_proj.weight'), np.float32)
                kvb = self._put(w.reshape(self.heads, self.nope + self.vdim, self.rank))
            L['kvb'] = kvb
            if self.indexer_types[i] == 'full':
                L['wq_b'] = self._proj(a + '.indexer.wq_b', self.ih * self.idim, self.q_lora)
                L['wk'] = self._proj(a + '.indexer.wk', self.idim, H)
                L['k_norm_w'] = self._vec(a + '.indexer.k_norm.weight', self.idim)
                L['k_norm_b'] = self._vec(a + '.indexer.k_norm.bias', self.idim, ones=False)
                L['w_proj'] = self._proj(a + '.indexer.weights_proj', self.ih, H)
            m = p + '.mlp'
            if self.mlp_types[i] == 'dense':
                I = int(c['intermediate_size'])
                L['mlp'] = (self._proj(m + '.gate_proj', I, H), self._proj(m + '.up_proj', I, H),
                            self._proj(m + '.down_proj', H, I))
            elif self._moe_factory is not None:
                L['moe'] = self._moe_factory(i, self)
            else:
                L['moe'] = self._local_moe(m)
            self.layers.append(L)
        self.backend.stream.synchronize()

    def synthetic_experts(self, m, part, first, count, rows, cols):
        """Device stack of experts [first, first + count) of projection `part`
        of sparse layer `m`, each expert generated from its own name, so a
        rank's slice holds the same bytes as the whole stack would."""
        kind = self.source.kind(m + '.experts', (rows, cols))
        block, size, _ = LAYOUTS[kind]
        blocks = rows * cols // block
        buf = self._dev(count * blocks * size)
        for i, e in enumerate(range(first, first + count)):
            self.source.fill(self.lib, buf.ptr + i * blocks * size, kind, blocks, self.source.scale(kind, cols),
                             f'{m}.experts.{e}.{part}', False, self.s)
        return buf.ptr

    def _local_moe(self, m):
        c, H = self.config, self.hidden
        E, I = int(c['n_routed_experts']), int(c['moe_intermediate_size'])
        router = self._proj(m + '.gate', E, H)
        if router[1] != 0:
            raise ValueError('the router must be F32')
        bias = self._vec(m + '.gate.e_score_correction_bias', E, ones=False)
        stacks = []
        for part, (rows, cols) in (('gate_proj', (I, H)), ('up_proj', (I, H)), ('down_proj', (H, I))):
            if self._synthetic:
                kind = self.source.kind(m + '.experts', (rows, cols))
                stacks.append((self.synthetic_experts(m, part, 0, E, rows, cols), kind))
            else:
                raws = [self.source.packed_tensor(f'{m}.experts.{e}.{part}.weight') for e in range(E)]
                kinds = {r[1] for r in raws}
                if len(kinds) != 1:
                    raise ValueError('experts of one layer must share a format')
                stacks.append((self._put(np.concatenate([np.ascontiguousarray(r[0]).view(np.uint8) for r in raws])),
                               kinds.pop()))
        kind = stacks[0][1]
        shared = None
        if int(c.get('n_shared_experts', 1)) > 0:
            SI = I * int(c.get('n_shared_experts', 1))
            shared = tuple(self._proj(f'{m}.shared_experts.{part}', rows, cols)[0]
                           for part, (rows, cols) in (('gate_proj', (SI, H)), ('up_proj', (SI, H)),
                                                     ('down_proj', (H, SI))))
        return _LocalMoE(self, router[0], bias, kind, [s[0] for s in stacks], shared, E, H, I, self.k, self.scale_r)

    def _alloc_state(self):
        B, H, cap = self.B, self.hidden, self.capacity
        f = 4
        self.x = self._dev(f * B * H).ptr
        self.n = self._dev(f * B * H).ptr
        self.qa = self._dev(f * B * self.q_lora).ptr
        self.qr = self._dev(f * B * self.q_lora).ptr
        self.query = self._dev(f * B * self.heads * (self.nope + self.rot)).ptr
        self.comp = self._dev(f * B * (self.rank + self.rot)).ptr
        self.new_latent = self._dev(f * B * self.rank).ptr
        self.new_rope = self._dev(f * B * self.rot).ptr
        self.qi_raw = self._dev(f * B * self.ih * self.idim).ptr
        self.q_index = self._dev(f * B * self.ih * self.idim).ptr
        self.key_raw = self._dev(f * B * self.idim).ptr
        self.key_ln = self._dev(f * B * self.idim).ptr
        self.new_index = self._dev(f * B * self.idim).ptr
        self.hw_raw = self._dev(f * B * self.ih).ptr
        self.hw = self._dev(f * B * self.ih).ptr
        self.q_latent = self._dev(f * B * self.heads * self.rank).ptr
        self.q_rope = self._dev(f * B * self.heads * self.rot).ptr
        self.att = self._dev(f * B * self.heads * self.rank).ptr
        self.vout = self._dev(f * B * self.heads * self.vdim).ptr
        self.ffn = self._dev(f * B * H).ptr
        I = max([int(self.config.get('intermediate_size', 1))] + [1])
        self.g = self._dev(f * B * I).ptr
        self.u = self._dev(f * B * I).ptr
        self.act = self._dev(f * B * I).ptr
        self.logits = self._dev(f * B * self.vocab).ptr
        self.tokens = self._dev(4 * B).ptr
        self.full = self._dev(4).ptr
        for L, t in zip(self.layers, self.indexer_types):
            L['latents'] = self._dev(f * B * cap * self.rank).ptr
            L['rope_keys'] = self._dev(f * B * cap * self.rot).ptr
            L['index_keys'] = self._dev(f * B * cap * self.idim).ptr if t == 'full' else None
            L['lens'] = self._dev(4 * B)
            rt.call('glmvx_memset', L['lens'].ptr, 0, 4 * B, self.s)
            L['sel'] = self._dev(4 * B * self.topk).ptr if t == 'full' else None
        need = int(self.lib.glmvx_dsa_scratch_bytes(B, self.heads, self.rank, cap, self.topk))
        self.dsa_scratch, self.dsa_bytes = self._dev(need).ptr, need
        self.max_pos = cap
        cos, sin = rope_tables(self.rot, cap, self.theta)
        self.cos_tab, self.sin_tab = self._put(cos), self._put(sin)
        rt.call('glmvx_memset', self.full, 0, 4, self.s)
        rt.call('glmvx_memset', self.tokens, 0, 4 * B, self.s)
        self.host_tokens = rt.HostBuffer(4 * B)
        self.host_logits = None
        self.backend.stream.synchronize()

    # ------------------------------------------------------------- kernels
    def _check(self, code, name):
        rt.check(self.lib, code, name)

    def _linear(self, out, x, w):
        ptr, kind, rows, cols = w
        if kind == 0:
            self._check(self.lib.glmvx_matmul_nt(out, x, ptr, self.B, rows, cols, self.s), 'glmvx_matmul_nt')
        else:
            self._check(self.lib.glmvx_packed_gemm(kind, out, ptr, x, rows, cols, self.B, self.s), 'glmvx_packed_gemm')

    def _rmsnorm(self, out, x, w, n, eps, x_stride=None):
        self._check(self.lib.glmvx_rmsnorm_rows(out, x, w, self.B, n, x_stride or n, n, eps, self.s),
                    'glmvx_rmsnorm_rows')

    def _rope(self, out, x, pos, heads, d, tail, x_tok, x_head, x_off, out_tok, out_head, out_off=0):
        self._check(self.lib.glmvx_rope_rows(out, x, self.cos_tab, self.sin_tab, pos, self.B, heads, d, tail, x_tok,
                                             x_head, x_off, out_tok, out_head, out_off, self.max_pos, self.s),
                    'glmvx_rope_rows')

    def _attention(self, i, L, sel_prev):
        B, H, R, P, N, V = self.B, self.hidden, self.rank, self.rot, self.nope, self.vdim
        heads, IH, ID = self.heads, self.ih, self.idim
        pos = L['lens'].ptr  # cached rows per sequence = this token's position (read before the append)
        self._linear(self.qa, self.n, L['q_a'])
        self._rmsnorm(self.qr, self.qa, L['q_a_norm'], self.q_lora, 1e-6)
        self._linear(self.query, self.qr, L['q_b'])
        self._linear(self.comp, self.n, L['kv_a'])
        self._rmsnorm(self.new_latent, self.comp, L['kv_a_norm'], R, 1e-6, x_stride=R + P)
        self._rope(self.new_rope, self.comp, pos, 1, P, 0, R + P, 0, R, P, 0)
        full = self.indexer_types[i] == 'full'
        if full:
            self._linear(self.qi_raw, self.qr, L['wq_b'])
            self._rope(self.q_index, self.qi_raw, pos, IH, P, ID - P, IH * ID, ID, 0, IH * ID, ID)
            self._linear(self.key_raw, self.n, L['wk'])
            self._check(self.lib.glmvx_layernorm(self.key_ln, self.key_raw, L['k_norm_w'], L['k_norm_b'], B, ID,
                                                 C.c_float(1e-6), self.s), 'glmvx_layernorm')
            self._rope(self.new_index, self.key_ln, pos, 1, P, ID - P, ID, 0, 0, ID, 0)
            self._linear(self.hw_raw, self.n, L['w_proj'])
            self._check(self.lib.glmvx_scale(self.hw, self.hw_raw, C.c_float(np.float32(IH ** -0.5)), B * IH, self.s),
                        'glmvx_scale')
        self._check(self.lib.glmvx_absorb_query(self.q_latent, self.query, L['kvb'], B, heads, N, N + P, R, V,
                                                self.s), 'glmvx_absorb_query')
        self._rope(self.q_rope, self.query, pos, heads, P, 0, heads * (N + P), N + P, N, heads * P, P)
        self._check(self.lib.glmvx_dsa_append(L['latents'], L['rope_keys'], L['index_keys'], pos, self.new_latent,
                                              self.new_rope, self.new_index if full else None, B, self.capacity, R,
                                              P, ID if full else 0, self.full, self.s), 'glmvx_dsa_append')
        scale = float(np.float32((N + P) ** -0.5))
        if full:
            self._check(self.lib.glmvx_dsa_decode(
                self.att, L['sel'], self.q_latent, self.q_rope, self.q_index, self.hw, L['latents'], L['rope_keys'],
                L['index_keys'], pos, B, heads, R, P, IH, ID, self.capacity, self.topk,
                C.c_float(np.float32(ID ** -0.5)), C.c_float(scale), self.dsa_scratch, self.dsa_bytes, self.s),
                'glmvx_dsa_decode')
            sel = L['sel']
        else:
            self._check(self.lib.glmvx_dsa_attend(
                self.att, sel_prev, self.q_latent, self.q_rope, L['latents'], L['rope_keys'], pos, B, heads, R, P,
                self.capacity, self.topk, C.c_float(scale), self.dsa_scratch, self.dsa_bytes, self.s),
                'glmvx_dsa_attend')
            sel = sel_prev
        self._check(self.lib.glmvx_absorb_value(self.vout, self.att, L['kvb'], B, heads, N, R, V, self.s),
                    'glmvx_absorb_value')
        self._linear(self.ffn, self.vout, L['o'])  # attention output (ffn buffer reused)
        self._check(self.lib.glmvx_add(self.x, self.x, self.ffn, B * H, self.s), 'glmvx_add')
        return sel

    def _feed_forward(self, L):
        B, H = self.B, self.hidden
        self._rmsnorm(self.n, self.x, L['post_norm'], H, self.eps)
        if 'mlp' in L:
            gate, up, down = L['mlp']
            self._linear(self.g, self.n, gate)
            self._linear(self.u, self.n, up)
            self._check(self.lib.glmvx_swiglu(self.act, self.g, self.u, B * gate[2], self.s), 'glmvx_swiglu')
            self._linear(self.ffn, self.act, down)
        else:
            L['moe'].forward_device(self.ffn, self.n, B)
        self._check(self.lib.glmvx_add(self.x, self.x, self.ffn, B * H, self.s), 'glmvx_add')

    def attention_graph(self, layer=0):
        """A CUDA graph of layer `layer`'s attention sub-step alone (rmsnorm,
        projections, indexer, cache append, DSA attention, o_proj, residual)
        on the current hidden rows, for measuring it apart from the step."""
        L = self.layers[layer]
        g = rt.Graph(self.backend.stream)
        g.begin()
        try:
            self._rmsnorm(self.n, self.x, L['in_norm'], self.hidden, self.eps)
            self._attention(layer, L, None)
        finally:
            g.end()
        return g

    def _step_launches(self):
        """One decode step on the device: embed self.tokens, the layers, the
        logits, the argmax written back into self.tokens."""
        B, H = self.B, self.hidden
        ptr, kind, _, _ = self.embed
        self._check(self.lib.glmvx_embed_rows(self.x, ptr, kind, self.tokens, B, self.vocab, H, self.s),
                    'glmvx_embed_rows')
        sel = None
        for i, L in enumerate(self.layers):
            self._rmsnorm(self.n, self.x, L['in_norm'], H, self.eps)
            sel = self._attention(i, L, sel)
            self._feed_forward(L)
        self._rmsnorm(self.n, self.x, self.final_norm, H, self.eps)
        self._linear(self.logits, self.n, self.lm_head)
        self._check(self.lib.glmvx_argmax_rows(self.tokens, self.logits, B, self.vocab, self.s), 'glmvx_argmax_rows')

    # ---------------------------------------------------------------- API
    def step_graph(self):
        if self._graph is None:
            g = rt.Graph(self.backend.stream)
            g.begin()
            try:
                self._step_launches()
            finally:
                g.end()
            self._graph = g
        return self._graph

    def set_tokens(self, tokens):
        t = np.ascontiguousarray(np.asarray(tokens, np.int32).reshape(self.B))
        if t.min() < 0 or t.max() >= self.vocab:
            raise ValueError('token ids must be in the vocabulary')
        self.backend.stream.synchronize()  # the previous copy out of the pinned buffer has run
        view = self.host_tokens.view(np.int32, self.B)
        view[:] = t
        rt.call('glmvx_memcpy_htod', self.tokens, self.host_tokens.ptr, 4 * self.B, self.s)

    def read_tokens(self):
        rt.call('glmvx_memcpy_dtoh', self.host_tokens.ptr, self.tokens, 4 * self.B, self.s)
        self.backend.stream.synchronize()
        return self.host_tokens.view(np.int32, self.B).copy()

    def read_logits(self):
        out = np.empty((self.B, self.vocab), np.float32)
        self.backend.stream.synchronize()
        rt.call('glmvx_memcpy_dtoh', out.ctypes.data, self.logits, out.nbytes, self.s)
        self.backend.stream.synchronize()
        return out

    def step(self):
        """Advance every sequence by one token (graph replay)."""
        self.step_graph().launch()

    def check(self):
        """Raise on a device error (bounded wait, bad id) or a full cache."""
        self.backend.stream.synchronize()
        self.backend.device.check_device_error()
        flag = np.zeros(1, np.int32)
        rt.call('glmvx_memcpy_dtoh', flag.ctypes.data, self.full, 4, self.s)
        self.backend.stream.synchronize()
        if flag[0]:
            raise ValueError('a sequence exceeded the cache capacity')

    def generate(self, prompts, new_tokens, with_logits=False):
        """Greedy decode (glm_vx/generate.py:86-109 for each sequence):
        prompts [B][P] token ids, every sequence from an empty cache; returns
        (generated [B][new_tokens], logits of every sampled step or None)."""
        prompts = np.asarray(prompts, np.int64)
        if prompts.shape[0] != self.B or prompts.ndim != 2 or prompts.shape[1] < 1:
            raise ValueError('prompts must be [batch, length >= 1]')
        self.reset()
        for p in range(prompts.shape[1]):
            self.set_tokens(prompts[:, p])
            self.step()
        out, logits = [], []
        for i in range(new_tokens):
            if with_logits:
                logits.append(self.read_logits())
            out.append(self.read_tokens())
            if i + 1 < new_tokens:
                self.step()
        self.check()
        return np.stack(out, axis=1), (np.stack(logits, axis=1) if with_logits else None)

    def reset_slot(self, b):
        """Empty sequence b's caches in every layer (its length to 0)."""
        if not 0 <= b < self.B:
            raise ValueError('slot outside the batch')
        for L in self.layers:
            rt.call('glmvx_memset', L['lens'].ptr + 4 * b, 0, 4, self.s)

    def reset(self):
        """Empty every cache (lengths to 0)."""
        for L in self.layers:
            rt.call('glmvx_memset', L['lens'].ptr, 0, 4 * self.B, self.s)
        rt.call('glmvx_memset', self.full, 0, 4, self.s)

    def fill_caches(self, length, seed=1):
        """Stand-in for a prefill of `length` prompt tokens per sequence:
        every layer's caches get `length` random rows (latents, rope keys,
        index keys N(0,1)) and the lengths are set to `length`."""
        if not 0 < length < self.capacity:
            raise ValueError('length must leave room in the cache')
        B, cap = self.B, self.capacity
        for i, L in enumerate(self.layers):
            for key, dim in (('latents', self.rank), ('rope_keys', self.rot), ('index_keys', self.idim)):
                if L[key] is None:
                    continue
                n = B * cap * dim
                rt.check(self.lib, self.lib.glmvx_fill_random(L[key], 0, n, 7919 * seed + 31 * i + len(key), 1.0, 0,
                                                              self.s), 'glmvx_fill_random')
            lens = np.full(B, length, np.int32)
            L['lens'].upload(lens, self.s)
        self.backend.stream.synchronize()

    def close(self, barrier=None):
        """Free everything; with expert-parallel sparse layers pass the ranks'
        `barrier` (each layer's mailbox is freed only after every rank has
        unmapped it)."""
        self.backend.stream.synchronize()
        if self._graph is not None:
            self._graph.close()
            self._graph = None
        for L in getattr(self, 'layers', []):
            m = L.get('moe')
            if m is not None and hasattr(m, 'close'):
                m.close(barrier=barrier) if barrier is not None else m.close()
        if getattr(self, 'host_tokens', None) is not None:
            self.host_tokens.close()
            self.host_tokens = None
        for b in self._bufs:
            b.close()
        self._bufs = []


def expert_parallel_moe(rank, world, allgather):
    """moe_layer_factory for ResidentDecoder: every sparse layer as an
    ExpertParallelLayer (gpu/ep.py) holding this rank's experts
    [rank*E/world, (rank+1)*E/world) with the router and shared expert
    replicated, connected to the other ranks' layers through `allgather`
    (bytes -> [bytes per rank]).  Each rank decodes its own sequences (data-
    parallel attention); the ranks step together."""
    def factory(i, dec):
        from .ep import ExpertParallelLayer, experts_per_rank
        c, H = dec.config, dec.hidden
        E, I = int(c['n_routed_experts']), int(c['moe_intermediate_size'])
        per = experts_per_rank(E, world)
        m = f'model.layers.{i}.mlp'
        router = dec._proj(m + '.gate', E, H)
        if router[1] != 0:
            raise ValueError('the router must be F32')
        bias = dec._vec(m + '.gate.e_score_correction_bias', E, ones=False)
        stacks, kind = [], None
        for part, (rows, cols) in (('gate_proj', (I, H)), ('up_proj', (I, H)), ('down_proj', (H, I))):
            if dec._synthetic:
                kind = dec.source.kind(m + '.experts', (rows, cols))
                stacks.append(dec.synthetic_experts(m, part, rank * per, per, rows, cols))
            else:
                raws = [dec.source.packed_tensor(f'{m}.experts.{e}.{part}.weight') for e in range(rank * per,
                                                                                              (rank + 1) * per)]
                kind = raws[0][1]
                stacks.append(dec._put(np.concatenate([np.ascontiguousarray(r[0]).view(np.uint8) for r in raws])))
        shared = None
        if int(c.get('n_shared_experts', 1)) > 0:
            SI = I * int(c.get('n_shared_experts', 1))
            shared = tuple(dec._proj(f'{m}.shared_experts.{part}', rows, cols)[0]
                           for part, (rows, cols) in (('gate_proj', (SI, H)), ('up_proj', (SI, H)),
                                                     ('down_proj', (H, SI))))
        dec.backend.stream.synchronize()
        layer = ExpertParallelLayer(dec.backend, rank, world, router[0], bias, kind, *stacks, E, H, I, dec.k,
                                    dec.scale_r, shared=shared, max_tokens=dec.B, device_weights=True)
        layer.connect_ipc(allgather)
        return layer
    return factory


class _LocalMoE:
    """A sparse layer resident on this GPU (glmvx_moe_ffn) with its own workspace."""

    def __init__(self, dec, router, bias, kind, stacks, shared, experts, hidden, inter, k, scale):
        self.dec, self.lib = dec, dec.lib
        self.router, self.bias, self.kind = router, bias, kind
        self.gate, self.up, self.down = stacks
        self.shared = shared or (None, None, None)
        self.E, self.H, self.I, self.k, self.scale = experts, hidden, inter, k, scale
        need = int(self.lib.glmvx_moe_workspace_bytes(dec.B, hidden, inter, experts, k, int(shared is not None)))
        self.ws, self.ws_bytes = dec._dev(need).ptr, need

    def forward_device(self, y, x, tokens, ids=None, weights=None):
        rt.check(self.lib, self.lib.glmvx_moe_ffn(
            y, x, tokens, self.H, self.I, self.router, self.bias, self.E, self.k, self.scale, self.kind, self.gate,
            self.up, self.down, *self.shared, self.ws, self.ws_bytes, ids, weights, self.dec.s), 'glmvx_moe_ffn')
