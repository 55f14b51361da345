"""Multi-GPU plumbing for sequence-sharded runs: one process per GPU, each
owning whole sequences (their KV pools, block tables and plan), so the hot
path has no collective; ranks exchange only small stats after the timed
region. Backend-agnostic (NCCL on the GPUs, gloo in the CPU tests)."""
from __future__ import annotations

import numpy as np


def shard_range(rank: int, per_rank: int) -> range:
    """Global sequence indices owned by `rank` when every rank holds
    `per_rank` sequences (contiguous slices of the global list)."""
    return range(rank * per_rank, (rank + 1) * per_rank)


def balanced_shards(costs, nshards: int, per_shard: int) -> list:
    """Split len(costs) == nshards * per_shard items into `nshards` shards of
    exactly `per_shard` items with nearly equal total cost: items are taken
    longest first and each goes to the open shard (fewer than per_shard
    items) with the smallest total so far. Returns each shard's item
    indices in ascending order."""
    costs = np.asarray(costs, dtype=np.float64)
    if costs.shape[0] != nshards * per_shard:
        raise ValueError("need exactly nshards * per_shard items")
    totals = np.zeros(nshards)
    counts = np.zeros(nshards, dtype=np.int64)
    members = [[] for _ in range(nshards)]
    for i in np.argsort(-costs, kind="stable"):
        open_ = np.flatnonzero(counts < per_shard)
        s = int(open_[np.argmin(totals[open_])])
        members[s].append(int(i))
        totals[s] += costs[i]
        counts[s] += 1
    return [np.sort(np.asarray(m, dtype=np.int64)) for m in members]


def gather_floats(values, world: int, device: str = "cuda") -> np.ndarray:
    """All-gather a small float64 vector per rank -> [world, len(values)]."""
    import torch

    t = torch.tensor(values, dtype=torch.float64, device=device)
    if world == 1:
        return t.unsqueeze(0).cpu().numpy()
    import torch.distributed as dist

    out = [torch.empty_like(t) for _ in range(world)]
    dist.all_gather(out, t)
    return torch.stack(out).cpu().numpy()


def job_rate(units_per_rank, ms_per_rank) -> float:
    """Whole-job throughput: all ranks' units over the slowest rank's time
    (every rank's timed region is bracketed by the same barriers)."""
    units = float(np.sum(units_per_rank))
    ms = float(np.max(ms_per_rank))
    return units / (ms * 1e-3)
