"""Oracle (test infrastructure only): the reference's patched LLaMA attention
forward in fp32 on the host.

Restates ``StructureAwareAttentionWrapperTriton.forward``
(methods/sabrecoder/sabrecoder_llama_triton.py:270-319) in its default
"hybrid" mode: q/k/v projections, HF rotary embedding (:292-293), cache
update (:295-299), GQA ``repeat_interleave`` (:301-303), dense SDPA for
one-token decode (:305-308, :254-268) and the block-sparse prefill
(:309-313) computed by :func:`oracle.attention_oracle.sparse_prefill_fp32`
(or its gathered form, :func:`oracle.attention_oracle.sparse_prefill_fp32_gathered`,
when the lists are shared by all heads as in the reference).
"""

from __future__ import annotations

import torch
import torch.nn as nn

from .attention_oracle import sparse_prefill_fp32, sparse_prefill_fp32_gathered


class OracleAttention(nn.Module):
    def __init__(self, original_attn, block_indices, block_counts, block_size: int):
        super().__init__()
        self.layer_idx = getattr(original_attn, "layer_idx", 0)
        self.head_dim = original_attn.head_dim
        self.groups = original_attn.config.num_attention_heads // original_attn.config.num_key_value_heads
        self.q_proj, self.k_proj = original_attn.q_proj, original_attn.k_proj
        self.v_proj, self.o_proj = original_attn.v_proj, original_attn.o_proj
        self.bi, self.bc, self.block = block_indices, block_counts, block_size

    def forward(self, hidden_states, position_embeddings=None, attention_mask=None, past_key_value=None,
                cache_position=None, past_key_values=None, **kwargs):
        from transformers.models.llama.modeling_llama import apply_rotary_pos_emb
        cache = past_key_values if past_key_values is not None else past_key_value
        B, L = hidden_states.shape[:2]
        shp = (B, L, -1, self.head_dim)
        q = self.q_proj(hidden_states).view(shp).transpose(1, 2)
        k = self.k_proj(hidden_states).view(shp).transpose(1, 2)
        v = self.v_proj(hidden_states).view(shp).transpose(1, 2)
        cos, sin = position_embeddings
        q, k = apply_rotary_pos_emb(q, k, cos, sin)
        if cache is not None:
            k, v = cache.update(k, v, self.layer_idx, {"sin": sin, "cos": cos, "cache_position": cache_position})
        if self.groups > 1:
            k = k.repeat_interleave(self.groups, dim=1)
            v = v.repeat_interleave(self.groups, dim=1)
        if L == 1:
            o = torch.nn.functional.scaled_dot_product_attention(q, k, v, is_causal=False)
        else:
            shared = torch.as_tensor(self.bi).dim() == 3
            fn = sparse_prefill_fp32_gathered if shared else sparse_prefill_fp32
            o = fn(q, k, v, self.bi, self.bc, self.block).to(q.dtype)
        o = o.transpose(1, 2).reshape(B, L, -1)
        return self.o_proj(o), None


def patch_oracle(model, block_indices, block_counts, block_size: int):
    for layer in model.model.layers:
        layer.self_attn = OracleAttention(layer.self_attn, block_indices, block_counts, block_size)
    return model
