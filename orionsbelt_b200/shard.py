"""How the hot path is partitioned across GPUs (one process per GPU).

Every configuration of the path is a set of independent (batch, value head)
units: the recurrence never mixes sequences, and value head h only reads key
head h / (Hv/Hk).  So work splits with no exchange at all:

* by batch: rank r owns sequences [r*B/N, (r+1)*B/N) (configs 1, 2, 3), or,
  for weak scaling, its own B sequences;
* by value head: rank r owns a contiguous block of value heads whose key
  heads it owns completely (configs 0 and 2 when B < N), so q/k are never
  shared across ranks.

The only collective a run needs is the timing reduction (max over ranks).
"""
from __future__ import annotations


def batch_slice(global_batch: int, world: int, rank: int) -> tuple[int, int]:
    """[start, stop) of the sequences rank `rank` owns (contiguous, sizes differ by <= 1)."""
    if not 0 <= rank < world:
        raise ValueError("rank out of range")
    base, extra = divmod(global_batch, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def head_slice(heads_v: int, heads_k: int, world: int, rank: int) -> tuple[tuple[int, int], tuple[int, int]]:
    """Value-head and key-head ranges of rank `rank`: contiguous blocks of key
    heads with all the value heads that read them."""
    if heads_v % heads_k:
        raise ValueError("heads_v must be a multiple of heads_k")
    group = heads_v // heads_k
    k0, k1 = batch_slice(heads_k, world, rank)
    return (k0 * group, k1 * group), (k0, k1)


def rank_seed(base_seed: int, rank: int) -> int:
    """Seed of the inputs a rank generates for its own shard (weak scaling)."""
    return base_seed * 1000 + rank
