"""Token / request sharding of the PTQ forward across the GPUs of one box.

The path shards with no data-path collective: token rows are independent
given replicated weights and scales, and attention needs whole sequences, so
whole requests go to GPUs.  Requests are assigned greedily, longest first, to
the GPU with the fewest tokens so far (ties to the lower rank), then each
GPU's requests are packed back to back in their original order -- the packing
of the reference's pack_rows / pack_block_mask (tv/runtime/session.tkv:
3506-3566): segment offsets seg[0] = 0, seg[i+1] = seg[i] + len_i.

One process per GPU (torch.distributed, NCCL on the GPU box, gloo in the CPU
tests); collectives are used only for bookkeeping: the max over ranks of a
step time and the gather of per-rank token counts.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Sequence

import numpy as np


def shard_requests(lengths: Sequence[int], world: int) -> List[List[int]]:
    """Request indices per rank: longest-processing-time-first greedy
    assignment by token count.  Deterministic: equal lengths keep their
    index order, equal loads go to the lower rank."""
    if world < 1:
        raise ValueError("world size must be at least 1")
    lengths = [int(x) for x in lengths]
    if any(x < 1 for x in lengths):
        raise ValueError("every request needs at least one token")
    order = sorted(range(len(lengths)), key=lambda i: (-lengths[i], i))
    load = [0] * world
    out: List[List[int]] = [[] for _ in range(world)]
    for i in order:
        r = min(range(world), key=lambda k: (load[k], k))
        out[r].append(i)
        load[r] += lengths[i]
    for r in range(world):
        out[r].sort()
    return out


def pack_segments(lengths: Sequence[int]) -> np.ndarray:
    """Segment offsets of requests packed back to back: seg[0] = 0,
    seg[i + 1] = seg[i] + lengths[i] (int64)."""
    seg = np.zeros(len(lengths) + 1, np.int64)
    if len(lengths):
        seg[1:] = np.cumsum(np.asarray(lengths, np.int64))
    return seg


def ragged_lengths(n: int, total: int, lo: int, hi: int, seed: int) -> List[int]:
    """n request lengths drawn uniformly from [lo, hi] with a fixed seed, then
    adjusted deterministically (largest first / smallest first, one token at a
    time within [lo, hi]) so that they sum to `total` (config 4: 256 requests,
    U[32, 1024], 131072 tokens)."""
    if not (n * lo <= total <= n * hi):
        raise ValueError("total is out of reach of n lengths in [lo, hi]")
    rng = np.random.default_rng(seed)
    x = rng.integers(lo, hi + 1, n).astype(np.int64)
    diff = int(total - x.sum())
    # spread the difference evenly, then settle the remainder one by one
    while diff != 0:
        step = 1 if diff > 0 else -1
        room = (x < hi) if step > 0 else (x > lo)
        idx = np.flatnonzero(room)
        k = min(abs(diff), idx.size)
        if step > 0:
            pick = idx[np.argsort(x[idx], kind="stable")[:k]]
        else:
            pick = idx[np.argsort(-x[idx], kind="stable")[:k]]
        x[pick] += step
        diff -= step * k
    return [int(v) for v in x]


@dataclass
class RankPlan:
    """What one rank runs: its request indices (ascending), their lengths and
    the packed segment offsets."""
    rank: int
    requests: List[int]
    lengths: List[int]
    seg: np.ndarray

    @property
    def tokens(self) -> int:
        return int(self.seg[-1])


def plan(lengths: Sequence[int], world: int, rank: int) -> RankPlan:
    if not 0 <= rank < world:
        raise ValueError("rank out of range")
    req = shard_requests(lengths, world)[rank]
    lens = [int(lengths[i]) for i in req]
    return RankPlan(rank, req, lens, pack_segments(lens))


def max_over_ranks(value: float, device=None) -> float:
    """Max of a per-rank scalar (a step time) over the process group; the
    value itself without one."""
    import torch
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def gather_counts(count: int, device=None) -> List[int]:
    """Every rank's token count, in rank order."""
    import torch
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return [int(count)]
    t = torch.tensor([int(count)], dtype=torch.int64, device=device)
    out = [torch.zeros_like(t) for _ in range(dist.get_world_size())]
    dist.all_gather(out, t)
    return [int(x.item()) for x in out]
