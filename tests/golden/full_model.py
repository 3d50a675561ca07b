"""Seeded weights and requests of the BASELINE-scale decoder (config 3's model), shared by
the golden generator (which scores them with the reference's own code on the CPU) and the
GPU parity test (which scores them with this library). Neither side stores the 8 GB of
weights: both regenerate them here, tensor by tensor, from one CPU generator per tensor.

Model: a dense Qwen3 decoder with the 4B dims (hidden 2560, FFN 9728, 36 layers, 32 query /
8 key-value heads of 128, vocab 151936, tied lm_head). Linear and embedding weights are
N(0, 0.02) (the HF initialiser's std), norm weights N(1, 0.1), all rounded to bf16.
Requests: ids uniform over the vocab; 257 distinct readout rows (two labels, then 255
options, the reference readout's layout, v0.5/serving/lib/release_runtime.py:302-306) and
the softmax over the 255 options (:509-522)."""
from __future__ import annotations

import torch

HF_CONFIG = dict(hidden_size=2560, intermediate_size=9728, num_hidden_layers=36, num_attention_heads=32,
                 num_key_value_heads=8, head_dim=128, vocab_size=151936, rms_norm_eps=1e-6, rope_theta=1e6,
                 tie_word_embeddings=True, max_position_embeddings=40960)
SEED = 20261204
LENGTHS = (2048, 32768)
N_ROWS = 257
OPTION_SLICE = (2, 257)


def tensor_specs(layers: int = HF_CONFIG['num_hidden_layers']):
    """(HF state-dict name, shape, kind) in generation order; kind 'w' = N(0, 0.02), 'g' = N(1, 0.1)."""
    H, I = HF_CONFIG['hidden_size'], HF_CONFIG['intermediate_size']
    D = HF_CONFIG['head_dim']
    Q, KV = HF_CONFIG['num_attention_heads'] * D, HF_CONFIG['num_key_value_heads'] * D
    out = [('model.embed_tokens.weight', (HF_CONFIG['vocab_size'], H), 'w')]
    for i in range(layers):
        p = f'model.layers.{i}.'
        out += [(p + 'input_layernorm.weight', (H,), 'g'),
                (p + 'self_attn.q_proj.weight', (Q, H), 'w'),
                (p + 'self_attn.k_proj.weight', (KV, H), 'w'),
                (p + 'self_attn.v_proj.weight', (KV, H), 'w'),
                (p + 'self_attn.o_proj.weight', (H, Q), 'w'),
                (p + 'self_attn.q_norm.weight', (D,), 'g'),
                (p + 'self_attn.k_norm.weight', (D,), 'g'),
                (p + 'post_attention_layernorm.weight', (H,), 'g'),
                (p + 'mlp.gate_proj.weight', (I, H), 'w'),
                (p + 'mlp.up_proj.weight', (I, H), 'w'),
                (p + 'mlp.down_proj.weight', (H, I), 'w')]
    out.append(('model.norm.weight', (H,), 'g'))
    return out


def make_tensor(index: int, shape, kind: str, seed: int = SEED) -> torch.Tensor:
    """The index-th tensor of tensor_specs(), bf16 on the CPU (its own generator, so any
    subset can be made alone)."""
    g = torch.Generator().manual_seed(seed * 4096 + index)
    x = torch.randn(shape, generator=g)
    x = 1 + 0.1 * x if kind == 'g' else x * 0.02
    return x.to(torch.bfloat16)


def state(layers: int = HF_CONFIG['num_hidden_layers'], seed: int = SEED) -> dict:
    """The whole HF Qwen3ForCausalLM state dict (bf16, CPU); lm_head is the embedding itself."""
    out = {name: make_tensor(i, shape, kind, seed) for i, (name, shape, kind) in enumerate(tensor_specs(layers))}
    out['lm_head.weight'] = out['model.embed_tokens.weight']
    return out


def request(length: int, seed: int = SEED):
    """(ids int64 [length], readout row ids int64 [257]) of the request of that length."""
    g = torch.Generator().manual_seed(seed + length)
    rows = torch.randperm(HF_CONFIG['vocab_size'], generator=g)[:N_ROWS]
    ids = torch.randint(0, HF_CONFIG['vocab_size'], (length,), generator=g)
    return ids, rows
