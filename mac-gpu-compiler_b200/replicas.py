"""Multi-GPU runner: weight replicas, independent sequences sharded over ranks, no collective on
the data path.

Batch-1 decode of one sequence is not split across GPUs (a per-layer all-reduce would cost more
than the 1.2 GB weight read it saves). The box runs one process per GPU instead: every rank loads
its own copy of the weights and decodes its own share of the independent sequences
(the box workload, configs[4]: 64 sequences of a 130-id prompt plus 128 greedy steps). The only
cross-rank traffic is host-side bookkeeping around the timed region: a barrier before it, the
max of the ranks' device times after it, and the gathered token counts.

These helpers hold that bookkeeping so that it runs the same way under NCCL on the GPU box and
under gloo on CPU (the multi-process tests).
"""
from __future__ import annotations

from dataclasses import dataclass


def shard(n_items: int, world: int, rank: int) -> range:
    """The contiguous block of item indices rank `rank` owns when `n_items` independent items are
    split as evenly as possible over `world` ranks (the first n_items % world ranks get one more)."""
    if world <= 0 or not 0 <= rank < world or n_items < 0:
        raise ValueError("bad shard request")
    base, extra = divmod(n_items, world)
    start = rank * base + min(rank, extra)
    return range(start, start + base + (1 if rank < extra else 0))


def prompt_seed(sequence: int) -> int:
    """Seed of sequence `sequence`'s prompt ids (sequence 0 uses seed 1, the single-sequence
    workload's seed, so the 1-rank run decodes the same first sequence)."""
    return 1 + sequence


@dataclass
class RankTiming:
    tokens: int        # tokens this rank generated inside the timed region
    seconds: float     # this rank's device time of the timed region


def aggregate(timings: list[RankTiming]) -> dict:
    """Whole-box throughput: all ranks' tokens over the slowest rank's time (weak scaling)."""
    if not timings:
        raise ValueError("no ranks")
    slowest = max(t.seconds for t in timings)
    total = sum(t.tokens for t in timings)
    return {"tokens": total, "seconds": slowest, "tok_per_s": total / slowest if slowest > 0 else float("nan"),
            "ranks": len(timings)}


def reduce_timings(local: RankTiming, group=None) -> list[RankTiming]:
    """Every rank's (tokens, seconds), gathered on every rank through torch.distributed (NCCL on the
    GPU box, gloo on CPU); the identity without a process group."""
    if group is None:
        return [local]
    import torch
    import torch.distributed as dist
    backend = dist.get_backend()
    dev = torch.device("cuda", torch.cuda.current_device()) if backend == "nccl" else torch.device("cpu")
    mine = torch.tensor([float(local.tokens), local.seconds], dtype=torch.float64, device=dev)
    out = [torch.zeros_like(mine) for _ in range(dist.get_world_size())]
    dist.all_gather(out, mine)
    return [RankTiming(int(t[0].item()), float(t[1].item())) for t in out]
