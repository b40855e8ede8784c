"""Sharding of one attention layer across ranks (one process per GPU).

The block search and the attention of a query head read only that head's queries and its KV
head's keys and values, so a layer splits across ranks by KV-head groups with no exchange:
rank ``r`` of ``world`` owns KV heads ``[r*Hk/world, (r+1)*Hk/world)`` and their query heads
(query head ``h`` belongs to KV head ``h // (Hq/Hk)``, as in the reference's GQA indexing,
ops/flashprefill_native_forward.py:150-152).

With more ranks than KV heads (Qwen2.5-7B's 4 KV heads over 8 GPUs) each KV-head group is
further cut into contiguous query-block ranges, one per rank of the group (a 2-D split:
KV-head groups x query-block ranges).  Every query block of a head is still independent --
its block list depends only on its own queries and the pooled keys of earlier blocks -- so
the ranges need no exchange either; each rank holds its group's whole K/V and runs
``fpb_prefill_dense_rows`` over its range.  The ranges are balanced on an estimate of the
work of each query block: the search scans qb + 1 pooled keys, and the attention costs
about ``ATTN_PER_BLOCK`` times that per listed block; the listed blocks are estimated from
the structural rules (sinks, local window, whole last-N rows) plus a small density term.
"""
from __future__ import annotations

# Attention cost of one listed block relative to the search cost of one scanned pooled key,
# measured on one B200 at 128K tokens (search 0.82 ms over 16.8 M scanned (row, key block)
# pairs, attention 2.95 ms over 279 K listed blocks).
ATTN_PER_BLOCK = 216.0
# Listed blocks beyond the structural ones, as a fraction of the row length (measured density
# of threshold-selected blocks on the synthetic long-context layers is about 0.1-0.5%).
EXTRA_DENSITY = 2e-3


def head_shard(hq: int, hk: int, rank: int, world: int):
    """(hk0, hk1, hq0, hq1): the KV-head and query-head ranges owned by ``rank``."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    if hq % hk:
        raise ValueError(f"{hq} query heads do not group over {hk} KV heads")
    if hk % world:
        raise ValueError(f"{hk} KV heads do not split over {world} ranks")
    per = hk // world
    group = hq // hk
    hk0, hk1 = rank * per, (rank + 1) * per
    return hk0, hk1, hk0 * group, hk1 * group


def row_work(nb: int, sink: int = 2, window: int = 4, last_n: int = 2):
    """Estimated work of each query block of one head (search + attention), in units of one
    scanned pooled key."""
    out = []
    for qb in range(nb):
        if qb >= nb - last_n:
            listed = qb + 1
        else:
            s_end, w_lo = min(sink, qb + 1), max(0, qb - window + 1)
            w_n = qb + 1 - w_lo if window > 0 else 0
            listed = s_end + w_n - (max(0, s_end - w_lo) if window > 0 else 0)
            listed = min(qb + 1, listed + EXTRA_DENSITY * (qb + 1))
        out.append((qb + 1) + ATTN_PER_BLOCK * listed)
    return out


def row_ranges(nb: int, parts: int, sink: int = 2, window: int = 4, last_n: int = 2):
    """Boundaries b_0 = 0 < b_1 < ... < b_parts = nb cutting the query blocks into ``parts``
    contiguous ranges of about equal estimated work."""
    if not 1 <= parts <= nb:
        raise ValueError(f"cannot cut {nb} query blocks into {parts} ranges")
    w = row_work(nb, sink, window, last_n)
    total = sum(w)
    bounds, acc, k = [0], 0.0, 1
    for qb, x in enumerate(w):
        acc += x
        # close range k once it holds k/parts of the work, keeping one block per later range
        while k < parts and acc >= total * k / parts and qb + 1 <= nb - (parts - k):
            bounds.append(qb + 1)
            k += 1
    while len(bounds) < parts:
        bounds.append(nb - (parts - len(bounds)))
    bounds.append(nb)
    return bounds


def layer_shard(hq: int, hk: int, nb: int, rank: int, world: int, sink: int = 2, window: int = 4,
                last_n: int = 2):
    """(hk0, hk1, hq0, hq1, qb0, qb1): the heads and the query-block range owned by ``rank``.
    world <= hk: KV-head groups, every query block; world > hk (world a multiple of hk): one
    KV head per group of world/hk ranks, cut into balanced query-block ranges."""
    if world <= hk:
        return head_shard(hq, hk, rank, world) + (0, nb)
    if world % hk:
        raise ValueError(f"{world} ranks do not split over {hk} KV heads")
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    per = world // hk
    kv, part = divmod(rank, per)
    b = row_ranges(nb, per, sink, window, last_n)
    group = hq // hk
    return kv, kv + 1, kv * group, (kv + 1) * group, b[part], b[part + 1]
