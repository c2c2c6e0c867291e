"""Test infrastructure: write the synthetic packed checkpoint of refmodel.py
as a GLM-DSA GGUF checkpoint (llama.cpp tensor names and metadata, as the
reference's GGUFCheckpoint reads them: glm_vx/gguf_checkpoint.py:15-31,
45-71), in one file or a `-0000i-of-0000n` split set, with gguf-py's writer.

kv_b is stored the converted way, attn_k_b [heads][rank][nope] (the K half
transposed per head) and attn_v_b [heads][v][rank]; routed experts stacked
by expert id in ffn_<part>_exps; packed projections keep their GGML blocks.
"""
import numpy as np

from kernels.packed import LAYOUTS


def _meta(w, c, layers):
    rope = (c.get('rope_parameters') or {}).get('rope_theta', c.get('rope_theta', 8_000_000.0))
    ints = {'context_length': c['max_position_embeddings'], 'embedding_length': c['hidden_size'],
            'feed_forward_length': c['intermediate_size'], 'attention.head_count': c['num_attention_heads'],
            'attention.q_lora_rank': c['q_lora_rank'], 'attention.kv_lora_rank': c['kv_lora_rank'],
            'rope.dimension_count': c['qk_rope_head_dim'],
            'attention.key_length_mla': c['qk_nope_head_dim'] + c['qk_rope_head_dim'],
            'attention.value_length_mla': c['v_head_dim'], 'vocab_size': c['vocab_size'],
            'expert_count': c['n_routed_experts'], 'expert_used_count': c['num_experts_per_tok'],
            'expert_feed_forward_length': c['moe_intermediate_size'], 'expert_shared_count': c['n_shared_experts'],
            'leading_dense_block_count': c['first_k_dense_replace'],
            'attention.indexer.head_count': c['index_n_heads'], 'attention.indexer.key_length': c['index_head_dim'],
            'attention.indexer.top_k': c['index_topk'], 'expert_group_count': c['n_group'],
            'expert_group_used_count': c['topk_group'], 'expert_gating_func': 2, 'block_count': layers,
            'nextn_predict_layers': 0, 'attention.head_count_kv': 1,
            'attention.key_length': c['kv_lora_rank'] + c['qk_rope_head_dim'],
            'attention.value_length': c['kv_lora_rank']}
    for k, v in ints.items():
        w.add_uint32('glm-dsa.' + k, int(v))
    w.add_bool('glm-dsa.expert_weights_norm', True)
    for k, v in (('rope.freq_base', rope), ('expert_weights_scale', c['routed_scaling_factor']),
                 ('attention.layer_norm_rms_epsilon', c['rms_norm_eps'])):
        w.add_float32('glm-dsa.' + k, float(v))


def _packed(w, name, raw, kind, shape):
    import gguf
    rows, cols = shape
    if kind == 0:
        w.add_tensor(name, np.ascontiguousarray(raw).view(np.float32).reshape(rows, cols))
        return
    block, size, _ = LAYOUTS[kind]
    w.add_tensor(name, np.ascontiguousarray(raw).view(np.uint8).reshape(rows, cols // block * size),
                 raw_dtype=gguf.GGMLQuantizationType(kind))


def write_checkpoint(ckpt, config, path, split_max_tensors=0):
    """Write `ckpt` (refmodel.PackedCheckpoint of `config`) to `path`; with
    split_max_tensors the writer starts a new file after that many tensors.
    Returns the paths written."""
    import gguf
    c = config
    layers = int(c['num_hidden_layers'])
    w = gguf.GGUFWriter(str(path), 'glm-dsa', split_max_tensors=split_max_tensors)
    _meta(w, c, layers)
    d, p = ckpt.dense, ckpt.packed
    w.add_tensor('token_embd.weight', np.asarray(d['model.embed_tokens.weight'], np.float32))
    _packed(w, 'output.weight', *p['lm_head.weight'])
    w.add_tensor('output_norm.weight', np.asarray(d['model.norm.weight'], np.float32))
    heads, nope, rope, v, rank = (c['num_attention_heads'], c['qk_nope_head_dim'], c['qk_rope_head_dim'],
                                  c['v_head_dim'], c['kv_lora_rank'])
    for i in range(layers):
        hp, gp = f'model.layers.{i}', f'blk.{i}'
        a = hp + '.self_attn'
        w.add_tensor(gp + '.attn_norm.weight', d[hp + '.input_layernorm.weight'])
        w.add_tensor(gp + '.ffn_norm.weight', d[hp + '.post_attention_layernorm.weight'])
        for hf, gg in (('q_a_proj', 'attn_q_a'), ('q_b_proj', 'attn_q_b'), ('kv_a_proj_with_mqa', 'attn_kv_a_mqa'),
                       ('o_proj', 'attn_output')):
            _packed(w, f'{gp}.{gg}.weight', *p[f'{a}.{hf}.weight'])
        w.add_tensor(gp + '.attn_q_a_norm.weight', d[a + '.q_a_layernorm.weight'])
        w.add_tensor(gp + '.attn_kv_a_norm.weight', d[a + '.kv_a_layernorm.weight'])
        kvb = np.asarray(d[a + '.kv_b_proj.weight'], np.float32).reshape(heads, nope + v, rank)
        w.add_tensor(gp + '.attn_k_b.weight', np.ascontiguousarray(kvb[:, :nope, :].transpose(0, 2, 1)))
        w.add_tensor(gp + '.attn_v_b.weight', np.ascontiguousarray(kvb[:, nope:, :]))
        if a + '.indexer.wq_b.weight' in p:
            _packed(w, gp + '.indexer.attn_q_b.weight', *p[a + '.indexer.wq_b.weight'])
            _packed(w, gp + '.indexer.attn_k.weight', *p[a + '.indexer.wk.weight'])
            _packed(w, gp + '.indexer.proj.weight', *p[a + '.indexer.weights_proj.weight'])
            w.add_tensor(gp + '.indexer.k_norm.weight', d[a + '.indexer.k_norm.weight'])
            w.add_tensor(gp + '.indexer.k_norm.bias', d[a + '.indexer.k_norm.bias'])
        m = hp + '.mlp'
        if m + '.gate_proj.weight' in p:
            for part in ('gate', 'up', 'down'):
                _packed(w, f'{gp}.ffn_{part}.weight', *p[f'{m}.{part}_proj.weight'])
            continue
        _packed(w, gp + '.ffn_gate_inp.weight', *p[m + '.gate.weight'])
        w.add_tensor(gp + '.exp_probs_b.bias', d[m + '.gate.e_score_correction_bias'])
        E = int(c['n_routed_experts'])
        for part in ('gate', 'up', 'down'):
            pieces = [p[f'{m}.experts.{e}.{part}_proj.weight'] for e in range(E)]
            kind, (rows, cols) = pieces[0][1], pieces[0][2]
            block, size, _ = LAYOUTS[kind]
            stack = np.stack([np.ascontiguousarray(r).view(np.uint8).reshape(rows, cols // block * size)
                              for r, _, _ in pieces])
            w.add_tensor(f'{gp}.ffn_{part}_exps.weight', stack, raw_dtype=gguf.GGMLQuantizationType(kind))
            _packed(w, f'{gp}.ffn_{part}_shexp.weight', *p[f'{m}.shared_experts.{part}_proj.weight'])
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    from pathlib import Path
    return w.format_shard_names(Path(path))
