"""Multi-GPU layout of the decode path: one process per GPU, KV heads sharded.

Every KV group is independent along the whole path (its own cells, lists,
row list and attention), so N GPUs split the KV heads into N contiguous
shards and run with no collective on the data path.  The only cross-rank
traffic is measurement: a barrier around the timed region and the max of
each rank's device time (the job takes as long as its slowest rank).
"""
from __future__ import annotations

from typing import List, Sequence, Tuple

import torch


def shard_kv_heads(kv_heads: int, world_size: int, rank: int) -> Tuple[int, int]:
    """(first head, head count) of `rank`'s contiguous shard of `kv_heads`."""
    if world_size < 1 or not 0 <= rank < world_size:
        raise ValueError(f"rank {rank} outside world size {world_size}")
    if kv_heads % world_size != 0:
        raise ValueError(f"{kv_heads} KV heads do not shard over {world_size} ranks")
    per = kv_heads // world_size
    return rank * per, per


def max_over_ranks(values: Sequence[float], device: torch.device) -> List[float]:
    """Element-wise maximum of `values` over every rank of the default process
    group (the values themselves when no group is initialised or it has one
    rank).  Works with the nccl (CUDA tensors) and gloo (CPU) backends."""
    t = torch.tensor(list(values), dtype=torch.float64, device=device)
    if torch.distributed.is_available() and torch.distributed.is_initialized() and \
            torch.distributed.get_world_size() > 1:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return t.tolist()
