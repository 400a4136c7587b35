"""Expert-parallel load balancing with redundant experts (host-side planning).

The reference shards experts contiguously and every expert lives on exactly
one rank (reframework/parallel/ep.py:45-55).  Under skewed routing the rank
holding the hottest expert then bounds the layer's time.  With B200's 180 GB
per GPU a few extra expert copies cost little, so each rank keeps its
contiguous shard (its *primary* experts) plus ``redundant`` replica slots, and
each step's rows of an expert are split among the ranks holding it so that the
per-rank row counts even out.

Everything here is deterministic numpy, computed identically on every rank
from the same inputs (the global per-expert counts), so no extra
communication is needed to agree on the plan.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import List, Sequence, Tuple

import numpy as np

__all__ = ["place_experts", "split_rows", "Placement"]


@dataclass(frozen=True)
class Placement:
    """``slots[r]`` = global expert ids held by rank r (primaries first)."""

    slots: Tuple[Tuple[int, ...], ...]

    @property
    def world(self) -> int:
        return len(self.slots)

    def holders(self, num_experts: int) -> List[List[int]]:
        h: List[List[int]] = [[] for _ in range(num_experts)]
        for r, ss in enumerate(self.slots):
            for e in ss:
                h[e].append(r)
        return h


def _waterfill(n: int, base: List[int]) -> List[int]:
    """Split ``n`` rows over holders with current loads ``base`` so that the
    resulting loads are as equal as possible (integers; remainder to the
    lowest-loaded holders, ties by position)."""
    order = sorted(range(len(base)), key=lambda i: (base[i], i))
    loads = [base[i] for i in order]
    k = len(loads)
    while k > 1 and (n + sum(loads[:k])) / k <= loads[k - 1]:
        k -= 1
    level = (n + sum(loads[:k])) // k
    give = [max(0, level - loads[i]) if i < k else 0 for i in range(len(loads))]
    rem = n - sum(give)
    i = 0
    while rem > 0:
        give[i % k] += 1
        rem -= 1
        i += 1
    out = [0] * len(base)
    for pos, i in enumerate(order):
        out[i] = give[pos]
    return out


def split_rows(counts_all: np.ndarray, placement: Placement, rounds: int = 4) -> np.ndarray:
    """Rows of each expert assigned to each holder, balancing rows per rank.

    ``counts_all[r, e]`` = rows rank r routes to expert e this step.  Returns
    ``quota[e, h]`` (rows of expert e computed on rank h, zero where h does not
    hold e).  Single-holder experts are fixed; replicated experts start evenly
    split and are then repeatedly re-split (heaviest first) by water-filling
    against the load the other experts put on their holders, until nothing
    changes or ``rounds`` passes.
    """
    counts_all = np.asarray(counts_all, dtype=np.int64)
    E = counts_all.shape[1]
    R = placement.world
    total = counts_all.sum(axis=0)
    holders = placement.holders(E)
    quota = np.zeros((E, R), dtype=np.int64)
    replicated = []
    for e in range(E):
        hs = holders[e]
        if not hs:
            continue
        if len(hs) == 1:
            quota[e, hs[0]] = total[e]
        else:
            replicated.append(e)
            for i, h in enumerate(hs):
                quota[e, h] = total[e] // len(hs) + (1 if i < total[e] % len(hs) else 0)
    replicated.sort(key=lambda q: (-total[q], q))
    load = quota.sum(axis=0)
    for _ in range(rounds):
        changed = False
        for e in replicated:
            hs = holders[e]
            base = [int(load[h] - quota[e, h]) for h in hs]
            new = _waterfill(int(total[e]), base)
            for h, q in zip(hs, new):
                if quota[e, h] != q:
                    load[h] += q - quota[e, h]
                    quota[e, h] = q
                    changed = True
        if not changed:
            break
    return quota


def place_experts(load: Sequence[float], shards: Sequence[Tuple[int, int]], redundant: int) -> Placement:
    """Primaries from ``shards`` plus up to ``redundant`` replica slots per rank.

    Greedy on the balanced split: repeatedly take the busiest rank (under
    :func:`split_rows`), and copy its heaviest expert to the least-busy rank
    that has a free slot and does not hold that expert (ties: lower rank);
    stop when no copy lowers the busiest rank's load or no slot is free.
    """
    load = np.rint(np.asarray(load, dtype=np.float64)).astype(np.int64)
    E = load.size
    R = len(shards)
    slots = [list(range(a, b)) for a, b in shards]
    if sorted(e for s in slots for e in s) != list(range(E)):
        raise ValueError("shards must cover every expert exactly once")
    free = [redundant] * R
    cnt = load[None, :]

    def evaluate(ss):
        q = split_rows(cnt, Placement(tuple(tuple(s) for s in ss)))
        return q, q.sum(axis=0)

    q, rank_load = evaluate(slots)
    while any(free):
        busiest = int(np.argmax(rank_load))
        best = None
        for e in sorted(slots[busiest], key=lambda x: (-q[x, busiest], x)):
            cands = [r for r in range(R) if free[r] > 0 and e not in slots[r]]
            if not cands:
                continue
            r = min(cands, key=lambda c: (rank_load[c], c))
            trial = [list(s) for s in slots]
            trial[r].append(int(e))
            tq, tl = evaluate(trial)
            if tl.max() < rank_load.max() or (tl.max() == rank_load.max() and np.sort(tl)[-2] < np.sort(rank_load)[-2]):
                best = (r, int(e), tq, tl)
                break
        if best is None:
            break
        r, e, q, rank_load = best
        slots[r].append(e)
        free[r] -= 1
    return Placement(tuple(tuple(s) for s in slots))
