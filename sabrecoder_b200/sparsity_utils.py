"""Block-sparsity accounting over the causal-eligible (lower-triangle) region.

Same functions, arguments and results as the reference's utils/sparsity_utils.py;
density is active lower-triangle blocks / causal-eligible blocks, the
definition sabrecoder_llama_triton.py:140-160 also uses.
"""

from __future__ import annotations

import math
from typing import Optional, Tuple


def ceil_div(a: int, b: int) -> int:
    """utils/sparsity_utils.py:14-19."""
    a, b = int(a), int(b)
    if b <= 0:
        raise ValueError(f"ceil_div expects b>0, got b={b}")
    return -(-a // b)


def causal_total_positions(seq_len: int) -> int:
    """utils/sparsity_utils.py:22-26."""
    n = int(seq_len)
    return n * (n + 1) // 2 if n > 0 else 0


def causal_total_blocks(num_query_blocks: int, num_key_blocks: Optional[int] = None) -> int:
    """Causal-eligible blocks of an ``M x N`` block matrix (utils/sparsity_utils.py:29-46):
    rows grow by one block until they reach ``N``, then stay at ``N``."""
    m = int(num_query_blocks)
    n = m if num_key_blocks is None else int(num_key_blocks)
    if m <= 0 or n <= 0:
        return 0
    tri = min(m, n)
    return tri * (tri + 1) // 2 + max(0, m - n) * n


def _key_block_prefix(key_token_mask, seq_len: int, bs: int, num_blocks: int):
    """Inclusive prefix counts of key blocks holding at least one marked token."""
    flags = [0] * num_blocks
    if key_token_mask is not None:
        try:
            import torch

            if isinstance(key_token_mask, torch.Tensor):
                km = key_token_mask
                if km.dim() == 2 and km.shape[0] == 1:
                    km = km[0]
                if km.dim() != 1:
                    raise ValueError(f"key_token_mask must be 1D (or [1, L]), got shape={tuple(km.shape)}")
                if km.numel() != seq_len:
                    raise ValueError(f"key_token_mask length {km.numel()} != seq_len {seq_len}")
                key_token_mask = km.to(torch.bool).cpu().tolist()
        except ImportError:  # pragma: no cover
            pass
        if len(key_token_mask) != seq_len:
            raise ValueError(f"key_token_mask length {len(key_token_mask)} != seq_len {seq_len}")
        for i, v in enumerate(key_token_mask):
            if v:
                flags[i // bs] = 1
    prefix = [0]
    for f in flags:
        prefix.append(prefix[-1] + f)
    return prefix


def causal_active_blocks_window_plus_keys(seq_len: int, window_size: int, *, key_token_mask=None,
                                          block_size: int = 64) -> Tuple[int, int]:
    """Closed-form active-block count for ``window OR key-column`` patterns
    (utils/sparsity_utils.py:49-143). Returns ``(active, total_causal)``."""
    L = int(seq_len)
    if L <= 0:
        return 0, 0
    bs = int(block_size)
    nb = ceil_div(L, bs)
    total = nb * (nb + 1) // 2
    prefix = _key_block_prefix(key_token_mask, L, bs, nb)
    w = int(window_size)
    if w <= 0:
        return int(sum(prefix[qb + 1] for qb in range(nb))), int(total)
    span = ceil_div(w, bs)
    active = 0
    for qb in range(nb):
        start = max(0, qb - span)
        active += (qb - start + 1) + prefix[start]
    return int(active), int(total)


def causal_attended_positions_from_cap(seq_len: int, attend_cap: float) -> float:
    """utils/sparsity_utils.py:146-160: query ``i`` attends ``min(i, cap)`` keys."""
    if seq_len <= 0:
        return 0.0
    cap = max(0.0, min(float(attend_cap), float(seq_len)))
    full = int(math.floor(cap))
    return full * (full + 1) / 2.0 + (seq_len - full) * cap


def causal_attend_ratio_from_cap(seq_len: int, attend_cap: float) -> float:
    """utils/sparsity_utils.py:163-168."""
    denom = float(causal_total_positions(seq_len))
    if denom <= 0.0:
        return 0.0
    return min(max(causal_attended_positions_from_cap(seq_len, attend_cap) / denom, 0.0), 1.0)


def causal_sparsity_from_cap(seq_len: int, attend_cap: float) -> float:
    """utils/sparsity_utils.py:171-173."""
    return 1.0 - causal_attend_ratio_from_cap(seq_len, attend_cap)
