"""Oracle (test infrastructure only): fp32 CPU restatement of block-sparse
prefill and decode attention.

Prefill follows ``_fwd_kernel_sabrecoder``
(methods/sabrecoder/sabrecoder_attention_triton.py:28-116): query block ``m``
attends to the listed key blocks ``n`` with token-level causal masking
``key <= query`` (:82-84), scale ``1/sqrt(D)`` (:67), and a fully masked row
outputs zeros (``l == 0 -> 1``, :112). It is written as a dense masked softmax
in fp32, which the reference kernel matches to 3.3e-7 in fp32 (its own golden
run is committed in tests/golden and checked by tests/test_oracle_golden.py).

Grouped-query attention follows the reference wrapper's ``repeat_interleave``
of K/V heads (methods/sabrecoder/sabrecoder_llama_triton.py:301-303): query
head ``h`` reads key/value head ``h // (Hq // Hkv)``.

Decode has no reference counterpart (the reference decodes densely,
sabrecoder_llama_triton.py:305-308); its restatement is the same masked
softmax for one query row per sequence over the KV cache, keeping keys in the
listed blocks with index ``< T``.

Only tests, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` use this module.
"""

from __future__ import annotations

import math
from typing import Optional, Sequence

import numpy as np
import torch


def _block_mask_from_lists(idx: torch.Tensor, cnt: torch.Tensor, nb: int) -> torch.Tensor:
    """bool ``[..., nb_q, nb]`` from index lists ``[..., nb_q, max]`` and counts
    ``[..., nb_q]``; entries past the count, negative or ``>= nb`` are ignored."""
    idx = idx.long()
    ar = torch.arange(idx.shape[-1])
    valid = (ar < cnt.long().unsqueeze(-1)) & (idx >= 0) & (idx < nb)
    m = torch.zeros(idx.shape[:-1] + (nb + 1,), dtype=torch.bool)
    m.scatter_(-1, torch.where(valid, idx, torch.full_like(idx, nb)), True)
    return m[..., :nb]


def sparse_prefill_fp32(q, k, v, block_indices, block_counts, block_size: int,
                        scale: Optional[float] = None, heads: Optional[Sequence[int]] = None,
                        row_chunk: int = 2048) -> torch.Tensor:
    """Block-sparse causal attention in fp32.

    q: ``[B, Hq, L, D]``; k, v: ``[B, Hkv, L, D]``;
    block_indices: ``[B, nb, max]`` (shared by all heads, as in the reference)
    or ``[B, Hq, nb, max]`` (per head); block_counts matching without the last
    dim. Returns fp32 ``[B, Hq, L, D]``, or ``[B, len(heads), L, D]`` for the
    listed query heads only when ``heads`` is given.

    Rows are processed ``row_chunk`` at a time against the keys up to the
    chunk's last row (causality), so memory stays bounded at long L; every
    row's softmax still spans all of its allowed keys at once."""
    q = torch.as_tensor(q)
    k = torch.as_tensor(k)
    v = torch.as_tensor(v)
    Bsz, Hq, L, D = q.shape
    Hkv = k.shape[1]
    g = Hq // Hkv
    nb = (L + block_size - 1) // block_size
    bi = torch.as_tensor(block_indices)
    bc = torch.as_tensor(block_counts)
    bm = _block_mask_from_lists(bi, bc, nb)  # [B, nb, nb] or [B, H, nb, nb]
    if bm.dim() == 3:
        bm = bm[:, None]
    sc = 1.0 / math.sqrt(D) if scale is None else scale
    hs = list(range(Hq)) if heads is None else [int(h) for h in heads]
    out = torch.empty(Bsz, len(hs), L, D, dtype=torch.float32)
    for b in range(Bsz):
        for oi, h in enumerate(hs):
            hk = h // g
            bmh = bm[b, h if bm.shape[1] > 1 else 0]
            kf = k[b, hk].float()
            vf = v[b, hk].float()
            for r0 in range(0, L, row_chunk):
                r1 = min(L, r0 + row_chunk)
                rows = torch.arange(r0, r1)
                keys = torch.arange(r1)
                # token (row, key) allowed: its block pair is listed and key <= row
                a = bmh[rows // block_size][:, keys // block_size] & (keys[None, :] <= rows[:, None])
                s = (q[b, h, r0:r1].float() @ kf[:r1].T) * sc
                s = s.masked_fill(~a, float("-inf"))
                mx = s.max(-1, keepdim=True).values
                mx = torch.where(torch.isinf(mx), torch.zeros_like(mx), mx)
                p = torch.exp(s - mx)
                l = p.sum(-1, keepdim=True)
                l = torch.where(l == 0, torch.ones_like(l), l)
                out[b, oi, r0:r1] = (p @ vf[:r1]) / l
    return out


def sparse_prefill_fp32_gathered(q, k, v, block_indices, block_counts, block_size: int,
                                 scale: Optional[float] = None) -> torch.Tensor:
    """The same attention as :func:`sparse_prefill_fp32` for lists shared by
    all heads (``[B, nb, max]``, the reference's layout), computed only over
    the listed key blocks: for each query block the keys of its listed
    blocks ``<=`` the query block are gathered (in ascending block order) and
    every head's rows take a masked softmax over them (key ``<=`` row), in
    fp32, all heads at once. Fully masked rows give zeros. This is the
    kernel's own loop structure (``sabrecoder_attention_triton.py:70-112``:
    one query block against its listed key blocks), used where the dense
    form would be too slow on the host (whole-model runs at 12K+ tokens)."""
    q = torch.as_tensor(q)
    k = torch.as_tensor(k)
    v = torch.as_tensor(v)
    Bsz, Hq, L, D = q.shape
    Hkv = k.shape[1]
    g = Hq // Hkv
    nb = (L + block_size - 1) // block_size
    bi = torch.as_tensor(block_indices)
    bc = torch.as_tensor(block_counts)
    if bi.dim() != 3:
        raise ValueError("sparse_prefill_fp32_gathered: lists must be shared by all heads, [B, nb, max]")
    bm = _block_mask_from_lists(bi, bc, nb)  # [B, nb, nb]
    sc = 1.0 / math.sqrt(D) if scale is None else scale
    out = torch.zeros(Bsz, Hq, L, D, dtype=torch.float32)
    for b in range(Bsz):
        kf = k[b].float().repeat_interleave(g, dim=0) if g > 1 else k[b].float()
        vf = v[b].float().repeat_interleave(g, dim=0) if g > 1 else v[b].float()
        for qb in range(nb):
            r0, r1 = qb * block_size, min(L, (qb + 1) * block_size)
            kbs = torch.nonzero(bm[b, qb, :qb + 1]).flatten()
            if kbs.numel() == 0:
                continue
            keys = (kbs[:, None] * block_size + torch.arange(block_size)[None, :]).flatten()
            keys = keys[keys < L]
            rows = torch.arange(r0, r1)
            a = keys[None, :] <= rows[:, None]
            s = (q[b, :, r0:r1].float() @ kf[:, keys].transpose(-1, -2)) * sc  # [H, rows, keys]
            s = s.masked_fill(~a, float("-inf"))
            mx = s.max(-1, keepdim=True).values
            mx = torch.where(torch.isinf(mx), torch.zeros_like(mx), mx)
            p = torch.exp(s - mx)
            l = p.sum(-1, keepdim=True)
            l = torch.where(l == 0, torch.ones_like(l), l)
            out[b, :, r0:r1] = (p @ vf[:, keys]) / l
    return out


def sparse_decode_fp32(q, k_cache, v_cache, block_indices, block_counts, seq_lens,
                       block_size: int, scale: Optional[float] = None) -> torch.Tensor:
    """One query row per sequence over the KV cache.

    q: ``[B, Hq, D]``; k_cache, v_cache: ``[B, Hkv, Tmax, D]``;
    block_indices: ``[B, max]`` or ``[B, Hkv, max]``; block_counts ``[B]`` or
    ``[B, Hkv]``; seq_lens ``[B]``: keys ``>= seq_lens[b]`` are masked.
    Returns fp32 ``[B, Hq, D]``."""
    q = torch.as_tensor(q).float()
    kc = torch.as_tensor(k_cache).float()
    vc = torch.as_tensor(v_cache).float()
    Bsz, Hq, D = q.shape
    Hkv, Tmax = kc.shape[1], kc.shape[2]
    g = Hq // Hkv
    nbk = (Tmax + block_size - 1) // block_size
    bi = torch.as_tensor(block_indices)
    bc = torch.as_tensor(block_counts)
    bm = _block_mask_from_lists(bi.unsqueeze(-2), bc.unsqueeze(-1), nbk).squeeze(-2)
    if bm.dim() == 2:
        bm = bm[:, None].expand(Bsz, Hkv, nbk)
    sc = 1.0 / math.sqrt(D) if scale is None else scale
    out = torch.zeros(Bsz, Hq, D, dtype=torch.float32)
    for b in range(Bsz):
        T = int(seq_lens[b])
        for h in range(Hq):
            hk = h // g
            keep = bm[b, hk].repeat_interleave(block_size)[:Tmax].clone()
            keep[T:] = False
            if not keep.any():
                continue
            s = (kc[b, hk][keep] @ q[b, h]) * sc
            p = torch.softmax(s, 0)
            out[b, h] = p @ vc[b, hk][keep]
    return out


def dense_masked_sdpa(q, k, v, block_mask_2d, block_size: int) -> torch.Tensor:
    """The reference's dense fallback arithmetic
    (sabrecoder_attention_triton.py:2061-2066): SDPA with the block mask
    expanded to tokens and ANDed with causal. Runs in the inputs' dtype on the
    host; used as the timed CPU baseline."""
    L = q.shape[-2]
    bm = torch.as_tensor(block_mask_2d).bool()
    tok = bm.repeat_interleave(block_size, 0).repeat_interleave(block_size, 1)[:L, :L]
    allowed = tok & torch.ones(L, L, dtype=torch.bool).tril()
    if k.shape[1] != q.shape[1]:
        g = q.shape[1] // k.shape[1]
        k = k.repeat_interleave(g, dim=1)
        v = v.repeat_interleave(g, dim=1)
    return torch.nn.functional.scaled_dot_product_attention(q, k, v, attn_mask=allowed)


def token_masked_prefill_fp32(q, k, v, visible) -> torch.Tensor:
    """Attention restricted to a token-level visibility matrix ``[L, L]`` (the
    reference's token-level kernel, sabrecoder_attention_triton.py:119-215),
    in fp32 with P rounded to the input dtype; rows with nothing visible give 0."""
    B, H, L, D = q.shape
    g = H // k.shape[1]
    kf = k.float().repeat_interleave(g, dim=1)
    vf = v.float().repeat_interleave(g, dim=1)
    s = torch.matmul(q.float(), kf.transpose(-1, -2)) / (D ** 0.5)
    vis = torch.as_tensor(visible, dtype=torch.bool)
    s = s.masked_fill(~vis, float("-inf"))
    m = s.amax(-1, keepdim=True)
    m = torch.where(torch.isinf(m), torch.zeros_like(m), m)
    p = torch.exp(s - m)
    l = p.sum(-1, keepdim=True)
    o = torch.matmul(p.to(q.dtype).float(), vf)
    return torch.where(l > 0, o / l.clamp_min(1e-30), torch.zeros_like(o))
