"""Stream sharding across GPUs: one process per GPU, independent streams, no data-path collective.

Streams share nothing in the machine (each has its own key/value store; every word depends only on its own
prefix, base2.py:102-114), so N GPUs each take a disjoint block of the streams with a full weight replica. The
process group (NCCL on GPUs, gloo in the CPU tests) is used only for a barrier and the max-over-ranks time.
"""
from __future__ import annotations

import os

import numpy as np


def rank_env():
    """(rank, world_size, local_rank) from the torchrun environment (1 process, rank 0, when absent)."""
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


def stream_ids(seed: int, streams_per_rank: int, prompt_len: int, rank: int, world: int, vocab: int) -> np.ndarray:
    """This rank's prompts: rows [rank*S, (rank+1)*S) of one uniform draw of shape [world*S, prompt_len] from
    numpy default_rng(seed) (so rank 0 of any world size holds the single-GPU config's streams)."""
    ids = np.random.default_rng(seed).integers(0, vocab, (streams_per_rank * world, prompt_len))
    return ids[rank * streams_per_rank:(rank + 1) * streams_per_rank]


def partition(n_streams: int, rank: int, world: int) -> tuple[int, int]:
    """This rank's half-open block [lo, hi) of n_streams streams split as evenly as possible over world ranks (a
    fixed total shared out: strong scaling; every stream computed once, on exactly one rank)."""
    base, extra = divmod(n_streams, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def max_over_ranks(x: float, dist=None, device=None) -> float:
    """The largest x over all ranks (the job's time is its slowest rank's)."""
    if dist is None or not dist.is_initialized() or dist.get_world_size() == 1:
        return float(x)
    import torch
    t = torch.tensor([float(x)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())
