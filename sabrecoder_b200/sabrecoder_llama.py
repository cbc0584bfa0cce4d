"""Drop-in LLaMA attention wrapper.

Counterpart of methods/sabrecoder/sabrecoder_llama_triton.py: the same
module-level state API (current code, precomputed blocks, call counters,
timing and sparsity statistics, :11-183), the same wrapper constructor
(:186-252) and ``patch_model_with_sabrecoder_attention_triton`` (:322-402).

Differences in how the work is done (results are the same):
* Q/K/V stay in the projection's ``[B, L, H, D]`` memory; the kernels take
  strided ``[B, H, L, D]`` views, and query head ``h`` reads KV head
  ``h // (Hq // Hkv)`` directly -- no ``repeat_interleave`` copies
  (reference :301-303).
* Prefill attention is the tcgen05 block-sparse kernel; decode attention is
  the split-K decode kernel, over all cached blocks (the reference's dense
  decode, :305-308) or, with ``use_sparse_for_generation``, over the
  structure row of the last prompt block plus every generated block.
* The output is written straight into ``[B, L, H, D]`` memory so the
  ``transpose().contiguous()`` before ``o_proj`` (:315-316) is free.
* Both cache keyword spellings are accepted: ``past_key_value`` (the
  reference) and ``past_key_values`` (transformers >= 4.56).
"""

from __future__ import annotations

import time
from typing import Optional, Tuple

import torch
import torch.nn as nn

from . import kernels as K
from .kv_cache import SabreKVCache
from .sabrecoder_attention import StructureAwareSparseAttention

_SPARSE_CALL_COUNT = 0
_DENSE_CALL_COUNT = 0
_CURRENT_CODE = None
_SPARSITY_STATS = {"total_blocks": 0, "active_blocks": 0, "num_samples": 0, "enabled": False}
_ATTENTION_TIMING = {"total_time": 0.0, "call_count": 0, "sparse_time": 0.0, "dense_time": 0.0,
                     "sparse_calls": 0, "dense_calls": 0, "enabled": False}
_PRECOMPUTED_BLOCK_INDICES = None
_PRECOMPUTED_BLOCK_COUNTS = None
_DECODE_LISTS: dict = {}


def set_current_code(code: str):
    global _CURRENT_CODE
    _CURRENT_CODE = code


def get_current_code() -> Optional[str]:
    return _CURRENT_CODE


def clear_current_code():
    global _CURRENT_CODE
    _CURRENT_CODE = None


def set_precomputed_blocks(block_indices, block_counts):
    """Store active-block lists reused by every layer's attention call."""
    global _PRECOMPUTED_BLOCK_INDICES, _PRECOMPUTED_BLOCK_COUNTS
    _PRECOMPUTED_BLOCK_INDICES = block_indices
    _PRECOMPUTED_BLOCK_COUNTS = block_counts
    _DECODE_LISTS.clear()


def get_precomputed_blocks():
    return _PRECOMPUTED_BLOCK_INDICES, _PRECOMPUTED_BLOCK_COUNTS


def clear_precomputed_blocks():
    global _PRECOMPUTED_BLOCK_INDICES, _PRECOMPUTED_BLOCK_COUNTS
    _PRECOMPUTED_BLOCK_INDICES = None
    _PRECOMPUTED_BLOCK_COUNTS = None
    _DECODE_LISTS.clear()


def get_attention_call_counts():
    return {"sparse": _SPARSE_CALL_COUNT, "dense": _DENSE_CALL_COUNT}


def reset_attention_call_counts():
    global _SPARSE_CALL_COUNT, _DENSE_CALL_COUNT
    _SPARSE_CALL_COUNT = 0
    _DENSE_CALL_COUNT = 0


def enable_attention_timing(enabled: bool = True):
    _ATTENTION_TIMING["enabled"] = enabled
    if enabled:
        reset_attention_timing()


def reset_attention_timing():
    for k in ("total_time", "sparse_time", "dense_time"):
        _ATTENTION_TIMING[k] = 0.0
    for k in ("call_count", "sparse_calls", "dense_calls"):
        _ATTENTION_TIMING[k] = 0


def get_attention_timing():
    s = dict(_ATTENTION_TIMING)
    s["avg_time"] = s["total_time"] / s["call_count"] if s["call_count"] else 0.0
    s["avg_sparse_time"] = s["sparse_time"] / s["sparse_calls"] if s["sparse_calls"] else 0.0
    s["avg_dense_time"] = s["dense_time"] / s["dense_calls"] if s["dense_calls"] else 0.0
    return s


def enable_sparsity_tracking(enabled: bool = True):
    _SPARSITY_STATS["enabled"] = enabled
    if enabled:
        _SPARSITY_STATS.update(total_blocks=0, active_blocks=0, num_samples=0)


def update_sparsity_stats(block_mask: torch.Tensor):
    """Accumulate causal-region density of a 2-D block mask (reference :140-160)."""
    if not _SPARSITY_STATS["enabled"]:
        return
    if block_mask.dim() != 2:
        raise ValueError(f"update_sparsity_stats expects a 2D block_mask, got shape={tuple(block_mask.shape)}")
    from .sparsity_utils import causal_total_blocks
    m, n = block_mask.shape
    _SPARSITY_STATS["total_blocks"] += causal_total_blocks(m, n)
    _SPARSITY_STATS["active_blocks"] += int(block_mask.tril(diagonal=0).sum().item())
    _SPARSITY_STATS["num_samples"] += 1


def update_sparsity_stats_from_blocks(total_blocks: int, active_blocks: int):
    if not _SPARSITY_STATS["enabled"]:
        return
    _SPARSITY_STATS["total_blocks"] += int(total_blocks)
    _SPARSITY_STATS["active_blocks"] += int(active_blocks)
    _SPARSITY_STATS["num_samples"] += 1


def get_sparsity_stats():
    s = dict(_SPARSITY_STATS)
    if s["total_blocks"] > 0:
        s["attend_ratio"] = s["active_blocks"] / s["total_blocks"]
        s["sparsity_ratio"] = 1.0 - s["attend_ratio"]
    else:
        s["attend_ratio"] = 0.0
        s["sparsity_ratio"] = 0.0
    return s


def decode_block_lists(prompt_len: int, total_len: int, block_size: int, device) -> Tuple[torch.Tensor, torch.Tensor]:
    """Key-block list for a decode step at cache length ``total_len``.

    Sparse mode (precomputed prompt lists present): the mask row of the last
    prompt block -- the chunk the completion continues, its window and all
    global key columns -- plus every block from the first block past the
    prompt up to the current one. Dense mode: all blocks."""
    key = (prompt_len, total_len, block_size, str(device))
    hit = _DECODE_LISTS.get(key)
    if hit is not None:
        return hit
    nbk = (total_len + block_size - 1) // block_size
    bi, bc = get_precomputed_blocks()
    if bi is not None and prompt_len > 0:
        nb_p = (prompt_len + block_size - 1) // block_size
        last = bi[:, nb_p - 1] if bi.dim() == 3 else bi[:, 0, nb_p - 1]
        cnt = bc[:, nb_p - 1] if bc.dim() == 2 else bc[:, 0, nb_p - 1]
        extra = torch.arange(nb_p, max(nbk, nb_p), device=device, dtype=torch.int32)
        B = last.shape[0]
        lst = torch.cat([last.to(device), extra.unsqueeze(0).expand(B, -1)], dim=1)
        cnts = cnt.to(device) + extra.numel()
        # entries past each row's count in `last` are -1 padding: compact them
        order = torch.argsort((lst < 0).to(torch.int8), dim=1, stable=True)
        lst = torch.gather(lst, 1, order).contiguous()
        hit = (lst, cnts.to(torch.int32).contiguous())
    else:
        lst = torch.arange(nbk, device=device, dtype=torch.int32).unsqueeze(0)
        hit = (lst, torch.tensor([nbk], dtype=torch.int32, device=device))
    _DECODE_LISTS[key] = hit
    return hit


class StructureAwareAttentionWrapper(nn.Module):
    """LLaMA attention replacement (reference sabrecoder_llama_triton.py:186-319)."""

    def __init__(self, original_attn, tokenizer, use_sparse_for_generation: bool = False, block_size: int = 64,
                 window_size: int = 64, num_prefix_tokens: int = 128, num_suffix_tokens: int = 256,
                 use_token_level_sparsity: bool = False, embedding_weight: Optional[torch.Tensor] = None,
                 global_last_k_chunks: int = 2, max_chunk_tokens: int = 0, use_chunk_similarity: bool = False,
                 chunk_similarity_top_percent: float = 0.1, chunk_similarity_max_tokens_per_chunk: int = 256,
                 chunk_similarity_max_neighbors: int = 8, use_crossfile_chunk_similarity: bool = False,
                 crossfile_chunk_similarity_top_percent: Optional[float] = None, topk_blocks: int = 0,
                 fused_prefill_projection: bool = False):
        super().__init__()
        self.fused_prefill_projection = bool(fused_prefill_projection)
        self.original_attn = original_attn
        self.tokenizer = tokenizer
        self.use_sparse_for_generation = use_sparse_for_generation
        self.window_size = window_size
        self.num_prefix_tokens = num_prefix_tokens
        self.num_suffix_tokens = num_suffix_tokens
        self.use_token_level_sparsity = use_token_level_sparsity
        self.block_size = int(block_size)
        self.config = original_attn.config
        self.layer_idx = getattr(original_attn, "layer_idx", 0)
        self.head_dim = original_attn.head_dim
        self.num_heads = self.config.num_attention_heads
        self.num_key_value_heads = self.config.num_key_value_heads
        self.num_key_value_groups = getattr(original_attn, "num_key_value_groups",
                                            self.num_heads // self.num_key_value_heads)
        self.scaling = original_attn.scaling
        self.attention_dropout = getattr(original_attn, "attention_dropout", 0.0)
        self.is_causal = True
        self.sparse_attn = StructureAwareSparseAttention(
            tokenizer=tokenizer, block_size=block_size, window_size=window_size,
            num_prefix_tokens=num_prefix_tokens, num_suffix_tokens=num_suffix_tokens,
            use_token_level_sparsity=use_token_level_sparsity, embedding_weight=embedding_weight,
            global_last_k_chunks=global_last_k_chunks, max_chunk_tokens=max_chunk_tokens,
            use_chunk_similarity=use_chunk_similarity, chunk_similarity_top_percent=chunk_similarity_top_percent,
            chunk_similarity_max_tokens_per_chunk=chunk_similarity_max_tokens_per_chunk,
            chunk_similarity_max_neighbors=chunk_similarity_max_neighbors,
            use_crossfile_chunk_similarity=use_crossfile_chunk_similarity,
            crossfile_chunk_similarity_top_percent=crossfile_chunk_similarity_top_percent,
            topk_blocks=topk_blocks)
        self.q_proj = original_attn.q_proj
        self.k_proj = original_attn.k_proj
        self.v_proj = original_attn.v_proj
        self.o_proj = original_attn.o_proj
        self._prompt_len = 0

    def _fused_decode_ok(self, hidden_states: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> bool:
        """Whether a one-token step can use the fused projection + rotary +
        KV-store kernel: plain bias-free projections with contiguous weights
        of the activations' dtype, and shapes the kernel takes."""
        projs = (self.q_proj, self.k_proj, self.v_proj)
        if any(not isinstance(m, nn.Linear) or m.bias is not None for m in projs):
            return False
        dt = hidden_states.dtype
        if dt not in (torch.bfloat16, torch.float16) or not hidden_states.is_cuda:
            return False
        if any(m.weight.dtype != dt or not m.weight.is_contiguous() or m.weight.device != hidden_states.device
               for m in projs):
            return False
        B, _, hidden = hidden_states.shape
        if B > 8 or hidden % 8 or B * hidden * 2 > 160 * 1024 or self.head_dim != 128:
            return False
        if not hidden_states.is_contiguous() or cos.dtype != dt or sin.dtype != dt:
            return False
        if cos.numel() != B * self.head_dim or sin.shape != cos.shape:
            return False
        return hidden_states.data_ptr() % 16 == 0 and all(m.weight.data_ptr() % 16 == 0 for m in projs)

    def _fused_prefill_ok(self, hidden_states: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
                          pooling: bool) -> bool:
        """Whether a prompt can use the fused projection + rotary + KV-store
        GEMM (sabre_qkv_proj_rope): opted in, plain bias-free projections of
        the activations' dtype, 128-wide heads, and, when pooling, one
        sequence or a length that is a multiple of 256."""
        if not self.fused_prefill_projection:
            return False
        projs = (self.q_proj, self.k_proj, self.v_proj)
        if any(not isinstance(m, nn.Linear) or m.bias is not None for m in projs):
            return False
        dt = hidden_states.dtype
        if dt not in (torch.bfloat16, torch.float16) or not hidden_states.is_cuda or self.head_dim != 128:
            return False
        if any(m.weight.dtype != dt or m.weight.device != hidden_states.device for m in projs):
            return False
        B, L, hidden = hidden_states.shape
        if hidden % 8 or not hidden_states.is_contiguous() or hidden_states.data_ptr() % 16:
            return False
        if cos.dtype != dt or sin.shape != cos.shape or cos.shape[-1] != 128:
            return False
        return not pooling or B == 1 or L % 256 == 0

    def _qkv_weight(self) -> torch.Tensor:
        """[Wq; Wk; Wv] as one contiguous tensor. Made once: the three
        projections' weights then become views of it, so no weight memory is
        duplicated and the decode path keeps reading the same values."""
        w = getattr(self, "_w_qkv", None)
        if w is None or w.data_ptr() != self.q_proj.weight.data_ptr():
            with torch.no_grad():
                w = torch.cat([self.q_proj.weight, self.k_proj.weight, self.v_proj.weight]).contiguous()
                nq, nk = self.q_proj.weight.shape[0], self.k_proj.weight.shape[0]
                self.q_proj.weight.data = w[:nq]
                self.k_proj.weight.data = w[nq:nq + nk]
                self.v_proj.weight.data = w[nq + nk:]
            self._w_qkv = w
        return w

    def forward(self, hidden_states: torch.Tensor, position_embeddings: Tuple[torch.Tensor, torch.Tensor] = None,
                attention_mask: Optional[torch.Tensor] = None, past_key_value=None,
                cache_position: Optional[torch.LongTensor] = None, past_key_values=None, **kwargs):
        global _SPARSE_CALL_COUNT, _DENSE_CALL_COUNT
        cache = past_key_values if past_key_values is not None else past_key_value
        B, L = hidden_states.shape[:2]
        D = self.head_dim
        cos, sin = position_embeddings
        qp = kp = None
        if L == 1 and self._fused_decode_ok(hidden_states, cos, sin):
            # One token per sequence: one kernel does the three projections,
            # the rotation and the K/V store.
            Hq = self.q_proj.weight.shape[0] // D
            Hkv = self.k_proj.weight.shape[0] // D
            w = (self.q_proj.weight, self.k_proj.weight, self.v_proj.weight)
            q = torch.empty(B, 1, Hq, D, dtype=hidden_states.dtype, device=hidden_states.device)

            def store(k_out, v_out, pos):
                K.qkv_rope_decode(hidden_states.view(B, -1), *w, cos.reshape(B, D), sin.reshape(B, D),
                                  q.view(B, Hq, D), k_out, v_out, pos)
        elif L > 1 and self._fused_prefill_ok(hidden_states, cos, sin,
                                              pooling=self.sparse_attn.topk_blocks > 0):
            # A prompt: one GEMM for the three projections whose epilogue
            # rotates q and k, stores K and V and pools the blocks.
            w_qkv = self._qkv_weight()
            Hq = self.q_proj.weight.shape[0] // D
            Hkv = self.k_proj.weight.shape[0] // D
            q = torch.empty(B, L, Hq, D, dtype=hidden_states.dtype, device=hidden_states.device)
            pool_block = self.block_size if self.sparse_attn.topk_blocks > 0 else 0

            def store(k_out, v_out, pos):
                nonlocal qp, kp
                qp, kp = K.qkv_proj_rope(hidden_states, w_qkv, cos, sin, q, k_out, v_out, pos0=pos,
                                         pool_block=pool_block if pos == 0 else 0)
        else:
            q = self.q_proj(hidden_states).view(B, L, -1, D)
            k = self.k_proj(hidden_states).view(B, L, -1, D)
            v = self.v_proj(hidden_states).view(B, L, -1, D)
            Hq, Hkv = q.shape[2], k.shape[2]
            # One kernel rotates q in place and writes rotated K and V rows;
            # a fresh prefill also gets the per-block pooled q/k the top-k
            # extension needs.
            pool_block = self.block_size if (L > 1 and self.sparse_attn.topk_blocks > 0) else 0

            def store(k_out, v_out, pos):
                nonlocal qp, kp
                _, qp, kp = K.rope_qkv(q, k, v, cos, sin, k_out, v_out, pos0=pos,
                                       pool_block=pool_block if pos == 0 else 0)
        # K and V rows go into [B, Hkv, T, D] storage: the cache's own buffers
        # when it is a SabreKVCache, else new rows handed to the cache's update.
        if isinstance(cache, SabreKVCache):
            kbuf, vbuf, pos0 = cache.slots(self.layer_idx, L)
            store(kbuf, vbuf, pos0)
            kh, vh = cache.advance(self.layer_idx, L)
        else:
            kn = torch.empty(B, Hkv, L, D, dtype=q.dtype, device=q.device)
            vn = torch.empty_like(kn)
            store(kn, vn, 0)
            kh, vh = kn, vn
            if cache is not None:
                kh, vh = cache.update(kn, vn, self.layer_idx,
                                      {"sin": sin, "cos": cos, "cache_position": cache_position})
        qh = q.transpose(1, 2)
        pooled = (qp, kp) if qp is not None and kh.shape[2] == L else None
        timing = _ATTENTION_TIMING["enabled"]
        if timing:
            torch.cuda.synchronize()
            t0 = time.perf_counter()
        if L == 1:
            _DENSE_CALL_COUNT += 0 if self.use_sparse_for_generation else 1
            _SPARSE_CALL_COUNT += 1 if self.use_sparse_for_generation else 0
            T = kh.shape[2]
            if self.use_sparse_for_generation and get_precomputed_blocks()[0] is not None:
                lst, cnt = decode_block_lists(self._prompt_len, T, self.block_size, q.device)
            else:
                lst, cnt = decode_block_lists(0, T, self.block_size, q.device)
            if lst.shape[0] != B:
                lst = lst.expand(B, -1).contiguous()
                cnt = cnt.expand(B).contiguous()
            seq = torch.full((B,), T, dtype=torch.int32, device=q.device)
            out = K.decode_bsa(q.view(B, Hq, D), kh, vh, lst, cnt, seq, self.block_size,
                               softmax_scale=self.scaling)
            attn = out.view(B, 1, Hq * D)
        else:
            _SPARSE_CALL_COUNT += 1
            self._prompt_len = kh.shape[2]
            # [B, L, H, D] memory: the [B, H, L, D] view the kernel writes
            # reshapes to [B, L, H*D] for o_proj without a copy.
            out = torch.empty(B, L, Hq, D, dtype=q.dtype, device=q.device)
            code = get_current_code()
            if code is not None and kh.shape[2] == L:
                self.sparse_attn(qh, kh, vh, code=code, attention_mask=attention_mask, out=out.transpose(1, 2),
                                 pooled=pooled)
            else:
                out.transpose(1, 2).copy_(self.sparse_attn(qh, kh, vh, code=None, attention_mask=attention_mask))
            attn = out.view(B, L, Hq * D)
        if timing:
            torch.cuda.synchronize()
            dt = time.perf_counter() - t0
            _ATTENTION_TIMING["total_time"] += dt
            _ATTENTION_TIMING["call_count"] += 1
            kind = "sparse" if L > 1 else "dense"
            _ATTENTION_TIMING[f"{kind}_time"] += dt
            _ATTENTION_TIMING[f"{kind}_calls"] += 1
        return self.o_proj(attn), None


def patch_model_with_sabrecoder_attention(model, tokenizer, use_sparse_for_generation: bool = False,
                                          block_size: int = 64, window_size: int = 64,
                                          num_prefix_tokens: int = 128, num_suffix_tokens: int = 256,
                                          use_token_level_sparsity: bool = False, global_last_k_chunks: int = 2,
                                          max_chunk_tokens: int = 0, use_chunk_similarity: bool = False,
                                          chunk_similarity_top_percent: float = 0.1,
                                          chunk_similarity_max_tokens_per_chunk: int = 256,
                                          chunk_similarity_max_neighbors: int = 8,
                                          use_crossfile_chunk_similarity: bool = False,
                                          crossfile_chunk_similarity_top_percent: Optional[float] = None,
                                          topk_blocks: int = 0, fused_prefill_projection: bool = False,
                                          verbose: bool = True):
    """Replace every ``layer.self_attn`` with the wrapper (reference :322-402).

    ``fused_prefill_projection=True`` runs each prompt's q/k/v projections,
    rotary embedding, KV store and block pooling as one GEMM kernel
    (sabre_qkv_proj_rope) instead of three cuBLAS projections followed by the
    fused RoPE/KV kernel; the results agree to the GEMMs' accumulation order
    (RoPE itself is bit-exact on either path)."""
    if verbose:
        mode = "Full Sparse" if use_sparse_for_generation else "Hybrid (Sparse Prefill, Dense Generation)"
        print(f"Applying SabreCoder B200 attention [{mode}] block={block_size} window={window_size} "
              f"prefix={num_prefix_tokens} suffix={num_suffix_tokens} last_k={global_last_k_chunks} "
              f"max_chunk_tokens={max_chunk_tokens} topk_blocks={topk_blocks}")
    emb = model.get_input_embeddings() if hasattr(model, "get_input_embeddings") else None
    emb_w = getattr(emb, "weight", None) if emb is not None else None
    if use_chunk_similarity and emb_w is None:
        raise ValueError("use_chunk_similarity=True requires model.get_input_embeddings().weight to be available.")
    count = 0
    for layer in model.model.layers:
        if hasattr(layer, "self_attn"):
            layer.self_attn = StructureAwareAttentionWrapper(
                layer.self_attn, tokenizer=tokenizer, use_sparse_for_generation=use_sparse_for_generation,
                block_size=block_size, window_size=window_size, num_prefix_tokens=num_prefix_tokens,
                num_suffix_tokens=num_suffix_tokens, use_token_level_sparsity=use_token_level_sparsity,
                embedding_weight=emb_w, global_last_k_chunks=global_last_k_chunks,
                max_chunk_tokens=max_chunk_tokens, use_chunk_similarity=use_chunk_similarity,
                chunk_similarity_top_percent=chunk_similarity_top_percent,
                chunk_similarity_max_tokens_per_chunk=chunk_similarity_max_tokens_per_chunk,
                chunk_similarity_max_neighbors=chunk_similarity_max_neighbors,
                use_crossfile_chunk_similarity=use_crossfile_chunk_similarity,
                crossfile_chunk_similarity_top_percent=crossfile_chunk_similarity_top_percent,
                topk_blocks=topk_blocks, fused_prefill_projection=fused_prefill_projection)
            count += 1
    if verbose:
        print(f"Replaced {count} attention layers with block-sparse B200 attention")
    model._sparse_attn_enabled = True
    model._sparse_attn_config = {
        "type": "sabrecoder_b200", "use_sparse_for_generation": use_sparse_for_generation,
        "block_size": block_size, "window_size": window_size, "num_prefix_tokens": num_prefix_tokens,
        "num_suffix_tokens": num_suffix_tokens, "use_token_level_sparsity": use_token_level_sparsity,
        "global_last_k_chunks": global_last_k_chunks, "max_chunk_tokens": max_chunk_tokens,
        "use_chunk_similarity": use_chunk_similarity, "chunk_similarity_top_percent": chunk_similarity_top_percent,
        "chunk_similarity_max_tokens_per_chunk": chunk_similarity_max_tokens_per_chunk,
        "chunk_similarity_max_neighbors": chunk_similarity_max_neighbors,
        "use_crossfile_chunk_similarity": use_crossfile_chunk_similarity,
        "crossfile_chunk_similarity_top_percent": crossfile_chunk_similarity_top_percent,
        "topk_blocks": topk_blocks, "fused_prefill_projection": fused_prefill_projection,
    }
    return model


# Names the reference uses for the same objects.
StructureAwareAttentionWrapperTriton = StructureAwareAttentionWrapper
patch_model_with_sabrecoder_attention_triton = patch_model_with_sabrecoder_attention
