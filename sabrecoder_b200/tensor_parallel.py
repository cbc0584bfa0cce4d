"""Head-parallel tensor parallelism for the largest model (one process per GPU).

The reference runs every model on one device. For the 33B architecture
(56 query / 8 KV heads of 128, hidden 7168, MLP 19200) the layers are split
over the ranks of one box the Megatron way:

* attention: ``q_proj``/``k_proj``/``v_proj`` keep the rows of this rank's
  heads (column-parallel; 7 query heads and their 1 KV head per rank at 8
  ranks, so the GQA group never straddles ranks), ``o_proj`` keeps the
  matching input columns (row-parallel) and its partial output is summed
  over the ranks with one all-reduce;
* MLP: ``gate_proj``/``up_proj`` keep a slice of the intermediate rows,
  ``down_proj`` the matching columns, followed by one all-reduce;
* embeddings, norms and ``lm_head`` stay replicated.

The block-sparse attention itself needs no communication: its block lists
are shared by all heads (structure part) or per head (top-k part, computed
from each rank's own heads), and each rank runs the prefill / decode kernels
on its local heads. The two all-reduces per layer are the only collectives,
issued through ``torch.distributed`` (NCCL over NVLink on the GPUs, gloo on
the host in tests).

Sequence parallelism (``shard_llama_(..., sequence_parallel=True)``, the
default) changes where the token-wise work runs during a prefill whose length
divides by the rank count: between the head-parallel parts each rank keeps
only its 1/world of the tokens, so the norms and residual adds (which the
plain scheme repeats on every rank over the whole prompt) are split too. Each
all-reduce becomes a reduce-scatter over tokens, and the input of the
attention and of the MLP is all-gathered, the same bytes on the links. Decode
steps and other lengths use the all-reduces.
"""

from __future__ import annotations

import types
from typing import Optional

import torch
import torch.nn as nn
import torch.nn.functional as F


class SeqParallelState:
    """Shared by the layers of one sharded model: whether the current forward
    runs sequence-parallel (decided by the first layer from the length)."""

    def __init__(self, rank: int, world: int, group=None):
        self.rank, self.world, self.group = rank, world, group
        self.active = False


def _gloo(group) -> bool:
    import torch.distributed as dist
    return dist.get_backend(group) == "gloo"


def gather_tokens(x: torch.Tensor, st: SeqParallelState) -> torch.Tensor:
    """``[B, l, H]`` token shards of all ranks -> ``[B, l * world, H]`` in rank order."""
    import torch.distributed as dist
    B, l, H = x.shape
    xt = x.transpose(0, 1).contiguous()  # [l, B, H]: rank blocks along dim 0
    if _gloo(st.group):
        parts = [torch.empty_like(xt) for _ in range(st.world)]
        dist.all_gather(parts, xt, group=st.group)
        out = torch.cat(parts, 0)
    else:
        out = torch.empty((l * st.world, B, H), dtype=x.dtype, device=x.device)
        dist.all_gather_into_tensor(out, xt, group=st.group)
    return out.transpose(0, 1) if B > 1 else out.view(1, l * st.world, H)


def scatter_sum_tokens(y: torch.Tensor, st: SeqParallelState) -> torch.Tensor:
    """``[B, L, H]`` partial sums -> this rank's ``[B, L / world, H]`` of their sum."""
    import torch.distributed as dist
    B, L, H = y.shape
    l = L // st.world
    yt = y.transpose(0, 1).contiguous()  # [L, B, H]
    if _gloo(st.group):  # the host backend has no reduce-scatter: sum, then keep the shard
        dist.all_reduce(yt, group=st.group)
        out = yt[st.rank * l:(st.rank + 1) * l]
    else:
        out = torch.empty((l, B, H), dtype=y.dtype, device=y.device)
        dist.reduce_scatter_tensor(out, yt, group=st.group)
    return out.transpose(0, 1) if B > 1 else out.view(1, l, H)


class RowParallelLinear(nn.Module):
    """``y = all_reduce_sum(x_local @ W_local^T)`` (+ replicated bias, added once);
    under an active :class:`SeqParallelState` the sum is reduce-scattered over
    tokens instead."""

    def __init__(self, weight: torch.Tensor, bias: Optional[torch.Tensor], group=None):
        super().__init__()
        self.weight = nn.Parameter(weight, requires_grad=False)
        self.bias = None if bias is None else nn.Parameter(bias, requires_grad=False)
        self.group = group
        self.in_features = weight.shape[1]
        self.out_features = weight.shape[0]
        self.sp: Optional[SeqParallelState] = None

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        import torch.distributed as dist
        y = F.linear(x, self.weight)
        if dist.is_available() and dist.is_initialized():
            if self.sp is not None and self.sp.active:
                y = scatter_sum_tokens(y, self.sp)
            else:
                dist.all_reduce(y, group=self.group)
        if self.bias is not None:
            y = y + self.bias
        return y


def _sp_layer_forward(layer, hidden_states, attention_mask=None, position_ids=None, past_key_values=None,
                      use_cache=False, position_embeddings=None, **kwargs):
    """A decoder layer (the transformers LlamaDecoderLayer steps) with its
    token-wise work on this rank's token shard; see the module docstring."""
    import torch.distributed as dist
    st = layer._sabre_sp
    if layer._sabre_sp_first:
        L = hidden_states.shape[1]
        st.active = dist.is_available() and dist.is_initialized() and L > 1 and L % st.world == 0
        if st.active:
            l = L // st.world
            hidden_states = hidden_states[:, st.rank * l:(st.rank + 1) * l]
    if not st.active:
        return layer._sabre_dense_forward(hidden_states, attention_mask=attention_mask, position_ids=position_ids,
                                          past_key_values=past_key_values, use_cache=use_cache,
                                          position_embeddings=position_embeddings, **kwargs)
    residual = hidden_states
    h = gather_tokens(layer.input_layernorm(hidden_states), st)
    h, _ = layer.self_attn(hidden_states=h, attention_mask=attention_mask, position_ids=position_ids,
                           past_key_values=past_key_values, use_cache=use_cache,
                           position_embeddings=position_embeddings, **kwargs)
    h = residual + h  # o_proj reduce-scattered back to this rank's tokens
    residual = h
    h = layer.mlp(gather_tokens(layer.post_attention_layernorm(h), st))
    h = residual + h
    if layer._sabre_sp_last:
        h = gather_tokens(h, st)
    return h


def _rows(linear: nn.Linear, start: int, stop: int) -> nn.Linear:
    w = linear.weight.data[start:stop]
    b = None if linear.bias is None else linear.bias.data[start:stop]
    out = nn.Linear(linear.in_features, stop - start, bias=b is not None, device="meta", dtype=w.dtype)
    out.weight = nn.Parameter(w.clone() if w.device.type != "meta" else w, requires_grad=False)
    if b is not None:
        out.bias = nn.Parameter(b.clone() if b.device.type != "meta" else b, requires_grad=False)
    return out


def _cols(linear: nn.Linear, start: int, stop: int, group) -> RowParallelLinear:
    w = linear.weight.data[:, start:stop]
    w = w.contiguous() if w.device.type != "meta" else torch.empty(w.shape, dtype=w.dtype, device="meta")
    b = None if linear.bias is None else linear.bias.data
    return RowParallelLinear(w, b, group)


def tp_shapes(config, world: int):
    """(local query heads, local KV heads, local MLP width); raises when the
    model does not split evenly over ``world`` ranks."""
    hq, hkv = config.num_attention_heads, config.num_key_value_heads
    inter = config.intermediate_size
    if hq % world or hkv % world:
        raise ValueError(f"{hq} query / {hkv} KV heads do not split over {world} ranks")
    if inter % world:
        raise ValueError(f"MLP width {inter} does not split over {world} ranks")
    return hq // world, hkv // world, inter // world


def shard_llama_(model, rank: int, world: int, group=None, sequence_parallel: bool = True):
    """Split every decoder layer of a transformers ``LlamaForCausalLM`` in
    place for ``rank`` of ``world`` (before or after the attention patch: the
    wrapper and the oracle both infer the head count from the projection
    widths). Works on real or meta parameters. ``sequence_parallel`` splits
    the token-wise work of prefills over the ranks as well."""
    if world == 1:
        return model
    cfg = model.config
    hq_l, hkv_l, inter_l = tp_shapes(cfg, world)
    D = getattr(cfg, "head_dim", None) or cfg.hidden_size // cfg.num_attention_heads
    for layer in model.model.layers:
        attn = layer.self_attn
        attn.q_proj = _rows(attn.q_proj, rank * hq_l * D, (rank + 1) * hq_l * D)
        attn.k_proj = _rows(attn.k_proj, rank * hkv_l * D, (rank + 1) * hkv_l * D)
        attn.v_proj = _rows(attn.v_proj, rank * hkv_l * D, (rank + 1) * hkv_l * D)
        attn.o_proj = _cols(attn.o_proj, rank * hq_l * D, (rank + 1) * hq_l * D, group)
        mlp = layer.mlp
        mlp.gate_proj = _rows(mlp.gate_proj, rank * inter_l, (rank + 1) * inter_l)
        mlp.up_proj = _rows(mlp.up_proj, rank * inter_l, (rank + 1) * inter_l)
        mlp.down_proj = _cols(mlp.down_proj, rank * inter_l, (rank + 1) * inter_l, group)
    if sequence_parallel:
        st = SeqParallelState(rank, world, group)
        layers = list(model.model.layers)
        for i, layer in enumerate(layers):
            layer.self_attn.o_proj.sp = st
            layer.mlp.down_proj.sp = st
            layer._sabre_sp = st
            layer._sabre_sp_first = i == 0
            layer._sabre_sp_last = i == len(layers) - 1
            layer._sabre_dense_forward = layer.forward
            layer.forward = types.MethodType(_sp_layer_forward, layer)
        model._sabre_sp = st
    model._sabre_tp = (rank, world)
    return model


@torch.no_grad()
def materialize_random_(model, device, seed: int = 0, std: float = 0.02, dtype=torch.bfloat16):
    """Give every meta parameter/buffer of ``model`` real storage on ``device``
    with seeded N(0, std) values (norm weights set to 1), so a sharded model
    of any size is built without ever holding the full weights. Non-meta
    buffers (rotary inverse frequencies) are moved as they are."""
    gen = torch.Generator(device=device).manual_seed(seed)
    for mod in model.modules():
        for name, p in list(mod.named_parameters(recurse=False)):
            if p.device.type == "meta":
                t = torch.empty(p.shape, dtype=dtype, device=device)
                if name == "weight" and p.dim() == 1:
                    t.fill_(1.0)
                else:
                    t.normal_(0.0, std, generator=gen)
                setattr(mod, name, nn.Parameter(t, requires_grad=False))
            else:
                setattr(mod, name, nn.Parameter(p.data.to(device=device, dtype=dtype), requires_grad=False))
        bufs = list(mod.named_buffers(recurse=False))
        if any(b.device.type == "meta" for _, b in bufs):
            # Computed buffers (the rotary embedding's inverse frequencies):
            # rebuild the module from its config on the real device.
            if not hasattr(mod, "config"):
                raise ValueError(f"meta buffers of {type(mod).__name__} cannot be rebuilt")
            fresh = type(mod)(mod.config, device=device)
            for name, b in fresh.named_buffers(recurse=False):
                mod.register_buffer(name, b, persistent=False)
            for key in ("attention_scaling",):
                if hasattr(fresh, key):
                    setattr(mod, key, getattr(fresh, key))
        else:
            for name, b in bufs:
                mod.register_buffer(name, b.to(device), persistent=False)
    return model
