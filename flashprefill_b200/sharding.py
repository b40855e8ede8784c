"""Head sharding of one attention layer across ranks (one process per GPU).

The block search and the attention of a query head read only that head's queries and its KV
head's keys and values, so a layer splits across ranks by KV-head groups with no exchange:
rank ``r`` of ``world`` owns KV heads ``[r*Hk/world, (r+1)*Hk/world)`` and their query heads
(query head ``h`` belongs to KV head ``h // (Hq/Hk)``, as in the reference's GQA indexing,
ops/flashprefill_native_forward.py:150-152).
"""
from __future__ import annotations


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
