"""Sharding of one PQ database over the GPUs of a node (one process per GPU) and the merge of per-shard results.

The database shards contiguously by id: rank r of N owns rows [r * ceil(n / N), min(n, (r + 1) * ceil(n / N))) and
reports global ids (its index's id_base is the shard's first row). Every rank searches all queries over its shard;
one exchange, an all-gather of the nq x k (dist, id) lists ([rank][query][k] int64 pairs), feeds the warp-merge
kernel, which keeps the k best by (dist, id). Ties break by global id, so the merged result is the single-GPU
result bit for bit.

`merge_fn` / `search_fn` are injected so the same host logic runs on GPUs (NCCL + vk_merge_topk_device) and in the
CPU tests (gloo + the oracle).
"""
from __future__ import annotations

import math
from dataclasses import dataclass


@dataclass(frozen=True)
class Shard:
    rank: int
    world: int
    lo: int
    hi: int

    @property
    def rows(self) -> int:
        return self.hi - self.lo


def shard_of(n: int, world: int, rank: int) -> Shard:
    if not (0 <= rank < world):
        raise ValueError(f"rank {rank} outside world {world}")
    per = math.ceil(n / world)
    lo = min(n, rank * per)
    return Shard(rank, world, lo, min(n, lo + per))


def gathered_layout(nq: int, k: int, world: int) -> dict:
    """Strides of the all-gathered [rank][query][k] buffer for vk_merge_topk_device."""
    return {"lists": world, "k_in": k, "query_stride": k, "list_stride": nq * k}


def gather_and_merge(local, gathered, nq: int, k: int, all_gather, merge) -> None:
    """local: this rank's [nq, k] results; gathered: [world, nq, k] buffer; all_gather(gathered, local) fills it
    (a collective: every rank calls it); merge(gathered, layout, out) writes the merged [nq, k] result."""
    all_gather(gathered, local)
    world = gathered.shape[0]
    merge(gathered, gathered_layout(nq, k, world))
