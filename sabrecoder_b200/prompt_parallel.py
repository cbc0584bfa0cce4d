"""Prompt-parallel work split over the GPUs of one box.

The reference evaluates prompts one after another on a single device
(run_eval.py:223-236 precomputes each prompt's block lists, then generates);
prompts are independent, so one process per GPU takes a share of them and no
collective touches the data path. The split is longest-processing-time first
(LPT): prompts sorted by length, each given to the rank with the least work so
far, ties to the lower rank -- deterministic, so every rank computes the same
assignment without communicating.

Host-side collectives are only used around the data path: gathering per-prompt
results to one rank, and the max-over-ranks elapsed time that whole-job
throughput is quoted against.
"""

from __future__ import annotations

from typing import Any, Callable, List, Optional, Sequence, Tuple


def assign_prompts(lengths: Sequence[int], world: int) -> List[List[int]]:
    """Prompt indices per rank (LPT by length, ties to the lower rank and the
    lower prompt index). Every prompt is assigned exactly once."""
    if world <= 0:
        raise ValueError(f"world size must be positive, got {world}")
    lengths = [int(x) for x in lengths]
    if any(x < 0 for x in lengths):
        raise ValueError("prompt lengths must be non-negative")
    order = sorted(range(len(lengths)), key=lambda i: (-lengths[i], i))
    loads = [0] * world
    out: List[List[int]] = [[] for _ in range(world)]
    for i in order:
        r = min(range(world), key=lambda j: (loads[j], j))
        loads[r] += lengths[i]
        out[r].append(i)
    return out


def prompts_for_rank(lengths: Sequence[int], rank: int, world: int) -> List[int]:
    """The prompt indices this rank processes."""
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of {world}")
    return assign_prompts(lengths, world)[rank]


def rank_loads(lengths: Sequence[int], world: int) -> List[int]:
    """Tokens per rank under :func:`assign_prompts`."""
    return [sum(int(lengths[i]) for i in idx) for idx in assign_prompts(lengths, world)]


def run_prompts(process: Callable[[int], Any], lengths: Sequence[int], rank: int, world: int,
                dist=None, dst: int = 0) -> Optional[List[Any]]:
    """Run ``process(i)`` for this rank's prompts and gather every result to
    rank ``dst`` in prompt order (``None`` on the other ranks). With
    ``dist=None`` (one process) all prompts run here."""
    mine = prompts_for_rank(lengths, rank, world)
    local = [(i, process(i)) for i in mine]
    if dist is None or world == 1:
        return [r for _, r in sorted(local, key=lambda t: t[0])]
    gathered: Optional[List[Any]] = [None] * world if rank == dst else None
    dist.gather_object(local, gathered, dst=dst)
    if rank != dst:
        return None
    merged: List[Tuple[int, Any]] = [t for part in gathered for t in part]
    merged.sort(key=lambda t: t[0])
    if [i for i, _ in merged] != list(range(len(lengths))):
        raise RuntimeError("prompt-parallel gather lost or duplicated prompts")
    return [r for _, r in merged]


def max_over_ranks(value: float, dist=None, device=None) -> float:
    """The maximum of ``value`` over all ranks (the job's elapsed time)."""
    if dist is None:
        return float(value)
    import torch
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())
