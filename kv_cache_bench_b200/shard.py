"""Host-side sharding of a batched decode step across the GPUs of one node.

Two strategies (every (sequence, KV head) is independent and split-K merges stay on one GPU, so a
step needs no exchange until its outputs are gathered):
  * by sequence: longest-processing-time bin packing of sequences by length (sort by length
    descending, give each to the least-loaded rank); each rank owns its sequences' pages;
  * by KV head: rank r owns KV heads [r*Hkv/N, (r+1)*Hkv/N) of every page and the query heads of
    those groups.
After the step the per-rank outputs are all-gathered (one collective) and put back in global order.
"""
from __future__ import annotations

from typing import List, Sequence

import numpy as np


def lpt_assign(lens: Sequence[int], n_ranks: int) -> List[List[int]]:
    """Sequence ids per rank, longest-first greedy onto the least-loaded rank (ties: lowest rank,
    then lowest sequence id). Each rank's list is in ascending id order."""
    if n_ranks < 1:
        raise ValueError("n_ranks must be >= 1")
    lens = np.asarray(lens, np.int64)
    order = sorted(range(lens.size), key=lambda b: (-int(lens[b]), b))
    load = [0] * n_ranks
    owned: List[List[int]] = [[] for _ in range(n_ranks)]
    for b in order:
        r = min(range(n_ranks), key=lambda i: (load[i], i))
        owned[r].append(b)
        load[r] += int(lens[b])
    return [sorted(o) for o in owned]


def imbalance(lens: Sequence[int], owned: List[List[int]]) -> float:
    """max rank load / mean rank load (1.0 is perfect)."""
    loads = [sum(int(lens[b]) for b in o) for o in owned]
    mean = sum(loads) / max(len(loads), 1)
    return max(loads) / mean if mean else 1.0


def kv_head_ranges(num_kv_heads: int, n_ranks: int) -> List[range]:
    """Contiguous KV-head blocks per rank; Hkv must be a multiple of the rank count."""
    if num_kv_heads % n_ranks:
        raise ValueError(f"{num_kv_heads} KV heads do not split evenly over {n_ranks} ranks")
    per = num_kv_heads // n_ranks
    return [range(r * per, (r + 1) * per) for r in range(n_ranks)]


def sequence_gather_index(owned: List[List[int]], pad_to: int) -> np.ndarray:
    """Index into the all-gathered [n_ranks * pad_to] rows that yields global sequence order."""
    n = sum(len(o) for o in owned)
    idx = np.empty(n, np.int64)
    for r, o in enumerate(owned):
        for i, b in enumerate(o):
            idx[b] = r * pad_to + i
    return idx


def merge_kv_head_shards(gathered: np.ndarray) -> np.ndarray:
    """[n_ranks][B][H/n][D] -> [B][H][D] (query heads of rank r are r*H/n ... (r+1)*H/n - 1)."""
    n, B, hr, D = gathered.shape
    return np.ascontiguousarray(np.transpose(gathered, (1, 0, 2, 3)).reshape(B, n * hr, D))
