"""Sequence-length balancing across data-parallel ranks
(reference ``lumenrl/utils/seqlen_balancing.py:27-152``).

``karmarkar_karp(costs, k)``: largest-differencing partition of items into
``k`` equal-count bins minimising the maximum bin cost; the cost of a
sequence of length L is ``24576 * L + L**2`` (linear GEMM work plus
quadratic attention work, the reference's weighting).  ``balance_batch``
returns a row permutation that gives every rank one contiguous slice.
"""

from __future__ import annotations

import heapq
from typing import Sequence


def seq_cost(length: int, linear_coef: int = 24576) -> int:
    return linear_coef * length + length * length


def karmarkar_karp(costs: Sequence[float], k: int, equal_size: bool = True) -> list[list[int]]:
    n = len(costs)
    if k <= 0:
        raise ValueError("k must be positive")
    if equal_size and n % k:
        raise ValueError(f"{n} items cannot be split into {k} equal-size partitions")
    order = sorted(range(n), key=lambda i: costs[i], reverse=True)
    heap = []
    cnt = 0
    if equal_size:
        # seed states with k items at a time (one per bin), then difference
        for s in range(0, n, k):
            group = order[s: s + k]
            bins = [[i] for i in group] + [[] for _ in range(k - len(group))]
            sums = [costs[i] for i in group] + [0.0] * (k - len(group))
            state = sorted(zip(sums, bins), key=lambda x: -x[0])
            spread = state[0][0] - state[-1][0]
            heapq.heappush(heap, (-spread, cnt, state))
            cnt += 1
    else:
        for i in order:
            state = [(costs[i], [i])] + [(0.0, []) for _ in range(k - 1)]
            heapq.heappush(heap, (-costs[i], cnt, state))
            cnt += 1
    while len(heap) > 1:
        _, _, a = heapq.heappop(heap)
        _, _, b = heapq.heappop(heap)
        # pair the heaviest bin of a with the lightest of b
        merged = [(a[j][0] + b[k - 1 - j][0], a[j][1] + b[k - 1 - j][1]) for j in range(k)]
        merged.sort(key=lambda x: -x[0])
        heapq.heappush(heap, (-(merged[0][0] - merged[-1][0]), cnt, merged))
        cnt += 1
    final = heap[0][2] if heap else [(0.0, []) for _ in range(k)]
    return [sorted(b) for _, b in final]


def balance_batch(lengths: Sequence[int], world: int) -> list[int]:
    parts = karmarkar_karp([seq_cost(int(l)) for l in lengths], world)
    return [i for p in parts for i in p]


def partition_stats(lengths: Sequence[int], parts: list[list[int]]) -> dict:
    loads = [sum(seq_cost(int(lengths[i])) for i in p) for p in parts]
    return {"balance/max_load": max(loads), "balance/min_load": min(loads),
            "balance/imbalance": max(loads) / max(min(loads), 1)}
