"""Preallocated KV cache for the patched model.

A transformers ``Cache`` whose per-layer K/V live in ``[B, Hkv, Tmax, D]``
buffers allocated once. Through the standard ``update()`` it behaves like
``DynamicCache`` (it copies the new rows in and returns views of the filled
prefix), so ``model.generate(past_key_values=SabreKVCache(...))`` works
unchanged. The attention wrapper skips that copy: it asks a layer for the
slots of the next rows (``slots``), lets the fused RoPE kernel write the
rotated K and the V rows straight into them, then commits the length
(``advance``). The reference's ``DynamicCache`` concatenates the whole cache
on every update (transformers' DynamicLayer.update); this cache writes only
the new rows.
"""

from __future__ import annotations

from typing import Optional, Tuple

import torch
from transformers.cache_utils import Cache, CacheLayerMixin


class SabreCacheLayer(CacheLayerMixin):
    is_compileable = False
    is_sliding = False

    def __init__(self, batch_size: int, num_kv_heads: int, head_dim: int, max_cache_len: int,
                 dtype: torch.dtype, device):
        super().__init__()
        self.max_cache_len = int(max_cache_len)
        self.max_batch_size = int(batch_size)
        self.dtype, self.device = dtype, torch.device(device)
        self.buf_k = torch.empty(batch_size, num_kv_heads, max_cache_len, head_dim, dtype=dtype, device=device)
        self.buf_v = torch.empty_like(self.buf_k)
        self.length = 0
        self.is_initialized = True
        self._views()

    def _views(self) -> Tuple[torch.Tensor, torch.Tensor]:
        self.keys = self.buf_k[:, :, : self.length]
        self.values = self.buf_v[:, :, : self.length]
        return self.keys, self.values

    def _room(self, n: int) -> None:
        if self.length + n > self.max_cache_len:
            raise ValueError(f"SabreKVCache is full: {self.length} + {n} > max_cache_len {self.max_cache_len}")

    def lazy_initialization(self, key_states: torch.Tensor, value_states: torch.Tensor) -> None:
        return None

    def update(self, key_states: torch.Tensor, value_states: torch.Tensor, *args, **kwargs):
        n = key_states.shape[-2]
        self._room(n)
        self.buf_k[:, :, self.length : self.length + n].copy_(key_states)
        self.buf_v[:, :, self.length : self.length + n].copy_(value_states)
        self.length += n
        return self._views()

    def slots(self, n: int) -> Tuple[torch.Tensor, torch.Tensor, int]:
        """Views of the next ``n`` rows to write directly, and their start position."""
        self._room(n)
        return self.buf_k, self.buf_v, self.length

    def advance(self, n: int) -> Tuple[torch.Tensor, torch.Tensor]:
        self.length += n
        return self._views()

    def get_seq_length(self) -> int:
        return self.length

    def get_mask_sizes(self, query_length: int) -> Tuple[int, int]:
        return self.length + query_length, 0

    def get_max_cache_shape(self) -> int:
        return self.max_cache_len

    def reset(self) -> None:
        self.length = 0
        self._views()

    def crop(self, max_length: int) -> None:
        if max_length < 0:
            max_length = self.length + max_length
        self.length = max(0, min(self.length, max_length))
        self._views()

    def reorder_cache(self, beam_idx: torch.LongTensor) -> None:
        idx = beam_idx.to(self.buf_k.device)
        self.buf_k.copy_(self.buf_k.index_select(0, idx))
        self.buf_v.copy_(self.buf_v.index_select(0, idx))
        self._views()


class SabreKVCache(Cache):
    """Preallocated cache: ``SabreKVCache(config, batch_size=1, max_cache_len=T)``
    or with explicit ``num_layers`` / ``num_kv_heads`` / ``head_dim``."""

    def __init__(self, config=None, *, batch_size: int = 1, max_cache_len: int, device="cuda",
                 dtype: torch.dtype = torch.bfloat16, num_layers: Optional[int] = None,
                 num_kv_heads: Optional[int] = None, head_dim: Optional[int] = None):
        if config is not None:
            num_layers = num_layers or config.num_hidden_layers
            num_kv_heads = num_kv_heads or config.num_key_value_heads
            head_dim = head_dim or getattr(config, "head_dim", None) or config.hidden_size // config.num_attention_heads
        if not (num_layers and num_kv_heads and head_dim):
            raise ValueError("SabreKVCache needs a config or num_layers/num_kv_heads/head_dim")
        layers = [SabreCacheLayer(batch_size, num_kv_heads, head_dim, max_cache_len, dtype, device)
                  for _ in range(num_layers)]
        super().__init__(layers=layers)

    def slots(self, layer_idx: int, n: int):
        return self.layers[layer_idx].slots(n)

    def advance(self, layer_idx: int, n: int):
        return self.layers[layer_idx].advance(n)
