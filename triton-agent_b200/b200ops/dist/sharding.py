"""Partitioning of the operator workloads across ranks.

rmsnorm rows, KV appends and paged decode are independent per row /
sequence: each rank owns a disjoint set and its own KV pages, so the data
path has no collective.  Decode sequences are balanced by their KV bytes
(greedy longest-first), not by count, because context lengths vary 16x.
quant_matmul is split by output columns (rows of W); its one exchange step
is an all-gather of the column blocks (collectives.py).
"""

from __future__ import annotations

from typing import Sequence


def shard_rows(n_rows: int, world: int, rank: int) -> slice:
    """Contiguous near-equal row range of `rank`."""
    base, extra = divmod(n_rows, world)
    start = rank * base + min(rank, extra)
    return slice(start, start + base + (1 if rank < extra else 0))


def shard_sequences(context_len: Sequence[int], world: int) -> list[list[int]]:
    """Assigns sequence indices to ranks, longest first onto the least-loaded
    rank (LPT), so per-rank KV bytes balance.  Deterministic: ties go to the
    lower rank, equal lengths keep index order."""
    order = sorted(range(len(context_len)), key=lambda i: (-int(context_len[i]), i))
    load = [0] * world
    parts: list[list[int]] = [[] for _ in range(world)]
    for i in order:
        r = min(range(world), key=lambda k: (load[k], k))
        parts[r].append(i)
        load[r] += max(0, int(context_len[i]))
    return [sorted(p) for p in parts]


def imbalance(context_len: Sequence[int], parts: list[list[int]]) -> float:
    """max rank load / mean rank load (1.0 = perfect)."""
    loads = [sum(max(0, int(context_len[i])) for i in p) for p in parts]
    mean = sum(loads) / len(loads)
    return max(loads) / mean if mean else 1.0


def column_shard(N: int, world: int, rank: int, align: int = 128) -> tuple[int, int]:
    """[n0, n1) of the output columns owned by `rank`: equal blocks rounded
    up to `align` columns (a GEMM tile), the last rank taking the remainder."""
    per = -(-N // world)
    per = -(-per // align) * align
    n0 = min(N, rank * per)
    return n0, min(N, n0 + per)
