"""Expert sharding across the GPUs of one node.

Each expert's gradient depends only on its own token slice, so the groups are partitioned into
contiguous ranges, one per rank, and every rank runs the kernel on its own slice with no
collective: LHS/RHS rows [off_a, off_b), group_offs rebased to start at 0, and C[a:b].
Range boundaries are chosen on the prefix sum of a per-group cost (tokens plus a fixed
per-group epilogue cost) so that ranks get equal work, not equal group counts.
The reference is single-device (README.md:18); this is the build's multi-GPU mode.
"""
from __future__ import annotations

import dataclasses

import numpy as np

# Per-group fixed cost in token-equivalents: writing C[g] (OUT_M x OUT_N bf16) at HBM speed
# takes about as long as the tensor cores need for this many tokens of the same group.
EPILOGUE_TOKEN_EQUIV = 256


@dataclasses.dataclass(frozen=True)
class Shard:
    rank: int
    g_begin: int
    g_end: int      # exclusive
    t_begin: int    # first token row (off_{g_begin})
    t_end: int      # off_{g_end}

    @property
    def groups(self) -> int:
        return self.g_end - self.g_begin

    @property
    def tokens(self) -> int:
        return self.t_end - self.t_begin


def partition(lens, world: int, epilogue_tokens: int = EPILOGUE_TOKEN_EQUIV) -> list[Shard]:
    """Split groups 0..G-1 into `world` contiguous ranges of near-equal cost.

    Boundary k is placed at the group edge whose cost prefix sum is closest to k/world of the
    total, kept strictly increasing where enough groups exist (a rank may get zero groups only
    when world > G)."""
    lens = np.asarray(lens, dtype=np.int64)
    G = lens.size
    if world < 1:
        raise ValueError("world must be >= 1")
    offs = np.zeros(G + 1, dtype=np.int64)
    offs[1:] = np.cumsum(lens)
    cost = np.zeros(G + 1, dtype=np.float64)
    cost[1:] = np.cumsum(lens.astype(np.float64) + float(epilogue_tokens))
    total = cost[-1]
    bounds = [0]
    for k in range(1, world):
        target = total * k / world
        b = int(np.searchsorted(cost, target))
        if b > 0 and abs(cost[b - 1] - target) <= abs(cost[min(b, G)] - target):
            b -= 1
        if G >= world:  # every rank keeps at least one group
            lo, hi = bounds[-1] + 1, G - (world - k)
        else:
            lo, hi = bounds[-1], G
        bounds.append(min(max(b, lo), hi))
    bounds.append(G)
    return [Shard(r, bounds[r], bounds[r + 1], int(offs[bounds[r]]), int(offs[bounds[r + 1]]))
            for r in range(world)]


def local_offsets(offs, shard: Shard) -> np.ndarray:
    """group_offs of a shard, rebased so its first group starts at token 0."""
    offs = np.asarray(offs, dtype=np.int64)
    return offs[shard.g_begin:shard.g_end + 1] - offs[shard.g_begin]


def imbalance(lens, shards: list[Shard], epilogue_tokens: int = EPILOGUE_TOKEN_EQUIV) -> float:
    """max rank cost / mean rank cost (1.0 = perfect)."""
    lens = np.asarray(lens, dtype=np.int64)
    costs = [float(lens[s.g_begin:s.g_end].sum()) + epilogue_tokens * s.groups for s in shards]
    mean = sum(costs) / len(costs)
    return max(costs) / mean if mean > 0 else 1.0
