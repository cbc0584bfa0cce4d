"""Precomputed block lists on disk.

The reference's evaluator builds every prompt's index lists once, keeps them
as ``{sample_index: (block_indices, block_counts)}`` and can save that dict
with ``torch.save`` / reload it with ``torch.load`` to skip the precompute
(methods/sabrecoder/run_eval.py:188-240 and :637-643, flag
``--precomputed_blocks_path``). The same file format is read and written here,
so lists built by either implementation can be used by the other: the
reference's rows are unordered (unstable argsort) and this library's are
ascending, and both kernels accept either.
"""

from __future__ import annotations

from typing import Callable, Dict, Iterable, Optional, Tuple

import torch

Blocks = Dict[int, Tuple[torch.Tensor, torch.Tensor]]


def _check(idx: int, bi: torch.Tensor, bc: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    if not isinstance(bi, torch.Tensor) or not isinstance(bc, torch.Tensor):
        raise TypeError(f"sample {idx}: block_indices and block_counts must be tensors")
    if bi.dim() not in (3, 4) or bc.dim() != bi.dim() - 1 or tuple(bc.shape) != tuple(bi.shape[:-1]):
        raise ValueError(f"sample {idx}: block_indices {tuple(bi.shape)} / block_counts {tuple(bc.shape)} "
                         "are not [B, (H,) nb, max_active] / [B, (H,) nb]")
    if bi.dtype.is_floating_point or bc.dtype.is_floating_point:
        raise TypeError(f"sample {idx}: block lists must be integer tensors")
    return bi.to(torch.int32), bc.to(torch.int32)


def save_precomputed_blocks(path: str, blocks: Blocks) -> None:
    """Write ``{sample: (block_indices, block_counts)}`` as the reference does
    (torch.save of host int32 tensors)."""
    out = {}
    for idx, (bi, bc) in blocks.items():
        bi, bc = _check(int(idx), bi, bc)
        out[int(idx)] = (bi.detach().cpu().contiguous(), bc.detach().cpu().contiguous())
    torch.save(out, path)


def load_precomputed_blocks(path: str, device: Optional[torch.device] = None) -> Blocks:
    """Read a file written by :func:`save_precomputed_blocks` or by the
    reference's evaluator; lists come back as int32 (on ``device`` if given)."""
    raw = torch.load(path, map_location="cpu", weights_only=True)
    if not isinstance(raw, dict):
        raise TypeError(f"{path}: expected a dict of sample -> (block_indices, block_counts)")
    out: Blocks = {}
    for idx, pair in raw.items():
        if not isinstance(pair, (tuple, list)) or len(pair) != 2:
            raise TypeError(f"{path}: sample {idx} is not a (block_indices, block_counts) pair")
        bi, bc = _check(int(idx), pair[0], pair[1])
        if device is not None:
            bi, bc = bi.to(device), bc.to(device)
        out[int(idx)] = (bi, bc)
    return out


def precompute_blocks(build: Callable[[int, object], Tuple[torch.Tensor, torch.Tensor, torch.Tensor]],
                      samples: Iterable[Tuple[int, object]]) -> Blocks:
    """The evaluator's precompute loop: ``build(idx, sample)`` returns a
    builder's ``(block_indices, block_counts, block_mask)`` for one prompt;
    the lists are kept per sample index."""
    out: Blocks = {}
    for idx, sample in samples:
        bi, bc, _ = build(idx, sample)
        out[int(idx)] = (bi.clone(), bc.clone())
    return out
