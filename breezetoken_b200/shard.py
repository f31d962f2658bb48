"""Sequence sharding across GPUs (one process per GPU, no data-path collective).

The Qwen3.5 decode path shards by independent sequences: every rank holds a
full replica of the weights, its own KV / GDN / conv state and its own CUDA
graph, and decodes its own batch of sequences.  The only cross-rank traffic
is timing: a barrier around the timed region and the max of the ranks'
times, so aggregate throughput is counted against the slowest rank.
"""

from __future__ import annotations

from typing import Sequence

import numpy as np
import torch


def rank_prompts(rank: int, batch: int, vocab: int, length: int) -> list[list[int]]:
    """Prompts of rank `rank`: sequence b is uniform ids seeded by rank*batch + b,
    so no two sequences of the job share a prompt and any rank can be re-run alone."""
    return [np.random.default_rng(rank * batch + b).integers(0, vocab, length).tolist() for b in range(batch)]


def max_over_ranks(values: Sequence[float], device: torch.device | str = "cpu") -> list[float]:
    """Element-wise max of `values` over all ranks of the default process group
    (the values themselves when no group of more than one rank is initialised)."""
    import torch.distributed as dist

    t = torch.tensor(list(values), dtype=torch.float64, device=device)
    if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return [float(x) for x in t.cpu()]


def aggregate_rate(units_per_rank: int, world: int, slowest_seconds: float) -> float:
    """Whole-job throughput: units of all ranks over the slowest rank's time."""
    return units_per_rank * world / slowest_seconds
