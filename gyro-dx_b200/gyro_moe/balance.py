"""Which experts an expert-parallel group should replicate (gx_replicate_experts).

With W ranks, rank r holds experts [r*NE/W, (r+1)*NE/W) of a layer. Skewed routing loads the rank
holding the popular experts. A replicated expert is served on every rank for that rank's own
tokens, so its load spreads evenly. Greedy policy: replicate experts in order of popularity until
the busiest rank's share is within `slack` of the even share, or `max_replicas` is reached.
"""
from __future__ import annotations

import numpy as np


def rank_loads(counts: np.ndarray, world: int, replicas=()) -> np.ndarray:
    """Slots each rank serves: its shard's unreplicated experts plus 1/W of every replica."""
    counts = np.asarray(counts, dtype=np.float64)
    per = counts.size // world
    own = counts.copy()
    rep = np.zeros_like(own, dtype=bool)
    rep[list(replicas)] = True
    spread = own[rep].sum() / world
    own[rep] = 0.0
    return own.reshape(world, per).sum(axis=1) + spread


def choose_replicas(counts: np.ndarray, world: int, max_replicas: int = 32, slack: float = 1.1) -> list[int]:
    counts = np.asarray(counts, dtype=np.float64)
    total = counts.sum()
    if world <= 1 or total == 0:
        return []
    chosen: list[int] = []
    for e in np.argsort(-counts, kind="stable"):
        if rank_loads(counts, world, chosen).max() <= slack * total / world or len(chosen) >= max_replicas:
            break
        if counts[e] == 0:
            break
        chosen.append(int(e))
    return chosen
