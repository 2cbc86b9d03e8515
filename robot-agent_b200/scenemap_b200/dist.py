"""Multi-GPU plumbing of the batch benchmark: maps shard across ranks, no collective on the
data path.

Rank r of W owns maps [r * M, (r + 1) * M) (per-map seeds = base seed mixed with the global map
index), so every rank generates and updates its own maps.  After the timed region the per-map
ApStats are gathered to every rank (one all_gather of an M x 16 int64 block; NCCL over NVLink
on the GPU box, gloo in the CPU tests), and the timed duration is the maximum over ranks (one
all_reduce(MAX)).  Every rank takes the same collective steps in the same order.
"""
from __future__ import annotations

import numpy as np


def rank_maps(rank: int, world: int, maps_per_rank: int) -> range:
    """Global indices of the maps rank `rank` owns."""
    if not (0 <= rank < world) or maps_per_rank <= 0:
        raise ValueError("bad rank / world / maps_per_rank")
    return range(rank * maps_per_rank, (rank + 1) * maps_per_rank)


def gather_stats(stats: np.ndarray, world: int, device=None) -> np.ndarray:
    """All ranks' per-map stats blocks (M x K int64 each) stacked in rank order."""
    import torch
    t = torch.from_numpy(np.ascontiguousarray(stats, np.int64))
    if device is not None:
        t = t.to(device)
    if world <= 1:
        return t.cpu().numpy()
    out = [torch.empty_like(t) for _ in range(world)]
    torch.distributed.all_gather(out, t)
    return torch.cat(out).cpu().numpy()


def max_over_ranks(values, world: int, device=None) -> list:
    """Element-wise maximum of a few float timings over all ranks."""
    import torch
    t = torch.tensor([float(v) for v in values], dtype=torch.float64, device=device)
    if world > 1:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return [float(v) for v in t.cpu()]
