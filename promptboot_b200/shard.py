"""Sequence sharding of the batched decode across ranks (one process per GPU).

The decode path partitions by sequence: rank r of a world of N owns a
contiguous block of the global sequences (`partition`: the batch split N ways,
strong scaling; `global_sequences`: a fixed S per rank, weak scaling), with its
own engine, model replica, KV and sampler states.
Nothing is exchanged on the hot path; the only collective is the max of the
ranks' device-timed durations after the timed region (and barriers around it).
These helpers are backend-agnostic (NCCL on GPUs, gloo in the CPU tests).
"""
from __future__ import annotations

import numpy as np

PROMPT_SEED = 0x5EED0000   # per-sequence prompt generator: default_rng(PROMPT_SEED + g)
VOCAB_PROMPT = 151643      # prompt ids uniform in [0, 151643)


def partition(total: int, rank: int, world: int) -> tuple[int, int]:
    """(first global index, count) of rank `rank`'s contiguous block when `total`
    sequences are split over `world` ranks (strong scaling: the first
    total % world ranks take one more)."""
    if not (0 <= rank < world) or total < world:
        raise ValueError("rank/world/total out of range")
    base, extra = divmod(total, world)
    count = base + (1 if rank < extra else 0)
    first = rank * base + min(rank, extra)
    return first, count


def global_sequences(rank: int, world: int, per_rank: int) -> np.ndarray:
    """Global indices of the sequences rank `rank` owns."""
    if not (0 <= rank < world) or per_rank <= 0:
        raise ValueError("rank/world/per_rank out of range")
    return rank * per_rank + np.arange(per_rank, dtype=np.int64)


def prompt_for(global_index: int, length: int) -> np.ndarray:
    """The seeded synthetic prompt of one global sequence (identical on every rank
    and at every world size)."""
    rng = np.random.default_rng(PROMPT_SEED + int(global_index))
    return rng.integers(0, VOCAB_PROMPT, length, dtype=np.uint32)


def prompts_for(rank: int, world: int, per_rank: int, length: int) -> np.ndarray:
    return np.stack([prompt_for(g, length) for g in global_sequences(rank, world, per_rank)])


def sampling_seed(global_index: int) -> int:
    """Per-sequence sampler seed: the global index (seed 0 takes the reference's
    replacement constant inside SamplingState)."""
    return int(global_index)


def barrier(world: int) -> None:
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(value: float, world: int, device: str = "cuda") -> float:
    """Maximum of a per-rank scalar (the timed duration) over all ranks."""
    if world == 1:
        return value
    import torch
    import torch.distributed as dist
    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def aggregate_throughput(tokens_per_rank: int, world: int, max_ms: float) -> float:
    """Whole-job tokens per second: every rank's tokens over the slowest rank's time."""
    return tokens_per_rank * world / (max_ms / 1000.0)
