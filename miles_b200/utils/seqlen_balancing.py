"""Sequence-length balancing: split samples into k groups of near-equal total tokens.

Used for --balance-data (equal sample counts per data-parallel rank, balanced token totals)
and --use-dynamic-batch-size (the fewest micro-batches that respect --max-tokens-per-gpu,
then balanced token totals across them). The reference does both with a Karmarkar-Karp
partition (miles/utils/seqlen_balancing.py:20-177, used by miles/ray/rollout.py:743-793 and
backends/training_utils/data.py:371-410).

Algorithm (largest differencing method, k-way, Karmarkar & Karp 1982): every partial solution
is k bins; start with one solution per item (that item alone in one bin) -- or, with equal
counts, one solution per run of k consecutive sorted items, one item per bin -- and repeatedly
merge the two solutions of largest spread (max bin sum - min bin sum) by pairing the heaviest
bin of one with the lightest bin of the other, until one solution is left. Ties are broken by
creation order, so the result is deterministic.
"""
from __future__ import annotations

import heapq


def _merge(a: list, b: list) -> list:
    """Pair a's bins (heaviest first) with b's bins (lightest first)."""
    a = sorted(a, key=lambda x: (-x[0], x[1]))
    b = sorted(b, key=lambda x: (x[0], x[1]))
    return [(sa + sb, ia + ib) for (sa, ia), (sb, ib) in zip(a, b)]


def karmarkar_karp(lengths: list[int], k: int, equal_size: bool = False) -> list[list[int]]:
    """Indices of `lengths` split into k lists (each sorted ascending) with near-equal sums.
    equal_size: every list gets len(lengths) / k items (len must divide evenly)."""
    n = len(lengths)
    if k <= 0:
        raise ValueError("k must be positive")
    if equal_size and n % k:
        raise ValueError(f"{n} items do not split into {k} equal-size groups")
    if n < k and not equal_size:
        out = [[i] for i in range(n)] + [[] for _ in range(k - n)]
        return out
    order = sorted(range(n), key=lambda i: (lengths[i], i))
    heap: list = []
    counter = 0

    def push(bins):
        nonlocal counter
        sums = [s for s, _ in bins]
        heapq.heappush(heap, (-(max(sums) - min(sums)), counter, bins))
        counter += 1

    if equal_size:
        for c in range(0, n, k):
            push([(lengths[i], [i]) for i in order[c:c + k]])
    else:
        for i in order:
            push([(lengths[i], [i])] + [(0, []) for _ in range(k - 1)])
    while len(heap) > 1:
        _, _, a = heapq.heappop(heap)
        _, _, b = heapq.heappop(heap)
        push(_merge(a, b))
    bins = heap[0][2]
    bins = sorted(bins, key=lambda x: (-x[0], min(x[1]) if x[1] else n))
    return [sorted(ix) for _, ix in bins]


def minimum_num_micro_batches(lengths: list[int], max_tokens: int) -> int:
    """Micro-batches needed so that each holds at most `max_tokens` tokens (first-fit
    decreasing; a single sample longer than the budget gets a micro-batch of its own)."""
    loads: list[int] = []
    for L in sorted(lengths, reverse=True):
        for b, s in enumerate(loads):
            if s + L <= max_tokens:
                loads[b] += L
                break
        else:
            loads.append(L)
    return len(loads)


def balanced_micro_batches(lengths: list[int], max_tokens: int, num_mbs: int | None = None) -> list[list[int]]:
    """--use-dynamic-batch-size: the fewest micro-batches that fit the budget (or `num_mbs`,
    e.g. the maximum over data-parallel ranks), token totals balanced across them."""
    k = num_mbs or minimum_num_micro_batches(lengths, max_tokens)
    return [b for b in karmarkar_karp(lengths, max(k, 1), equal_size=False) if b]


def rebalance_over_dp(data: dict, group) -> dict:
    """--balance-data: redistribute this rollout's samples over the data-parallel ranks so that
    every rank trains the same number of samples with near-equal token totals. Every
    per-sample list of `data` (same length as data["tokens"]) moves with its sample; other
    entries stay. Rewards are already group-normalised, so samples may leave their group."""
    import torch.distributed as dist

    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    n = len(data["tokens"])
    keys = [k for k, v in data.items() if isinstance(v, list) and len(v) == n]
    mine = {k: data[k] for k in keys}
    allp: list = [None] * world
    dist.all_gather_object(allp, mine, group=group)
    flat = {k: [x for p in allp for x in p[k]] for k in keys}
    lengths = [len(t) for t in flat["tokens"]]
    if len(lengths) % world:
        raise ValueError(f"--balance-data needs a sample count divisible by {world} DP ranks")
    part = karmarkar_karp(lengths, world, equal_size=True)[rank]
    out = dict(data)
    for k in keys:
        out[k] = [flat[k][i] for i in part]
    return out
