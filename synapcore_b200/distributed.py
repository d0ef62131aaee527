"""Multi-GPU layouts for the paged KV path (one process per GPU).

Sequence sharding (the default): sequences are dealt round-robin by id, each
rank owns its own pool, allocator and block tables, and decode attention
needs no communication — the aggregate is just the sum over ranks.

KV-head sharding (optional): every rank holds all sequences but only kv heads
[r*Hkv/n, (r+1)*Hkv/n) and the query heads that read them; after each
layer's attention the per-rank outputs [B, Hq/n, D] are all-gathered (NCCL
over NVLink) into [B, Hq, D]. The all-gather lands in a local buffer, so no
kernel ever reads another GPU's memory.

The reference has no multi-process code; these layouts are the B200 side's
way of scaling one box (8 GPUs).
"""
from __future__ import annotations

from typing import List, Optional, Sequence

import torch


def shard_of(seq_id: int, world: int) -> int:
    """Rank that owns sequence `seq_id` under round-robin sequence sharding."""
    return int(seq_id) % int(world)


def shard_sequences(seq_ids: Sequence[int], world: int, rank: int) -> List[int]:
    """The sequences rank `rank` owns, in their original order."""
    return [s for s in seq_ids if shard_of(s, world) == rank]


def head_range(num_kv_heads: int, world: int, rank: int) -> range:
    """kv heads owned by `rank` in KV-head-sharded mode (contiguous, equal)."""
    if num_kv_heads % world != 0:
        raise ValueError(f"{num_kv_heads} kv heads do not split evenly over {world} ranks")
    per = num_kv_heads // world
    return range(rank * per, (rank + 1) * per)


def query_head_range(num_q_heads: int, num_kv_heads: int, world: int, rank: int) -> range:
    """Query heads that read the kv heads of `rank` (q head h reads kv head h // G)."""
    g = num_q_heads // num_kv_heads
    kv = head_range(num_kv_heads, world, rank)
    return range(kv.start * g, kv.stop * g)


class HeadShardedOutput:
    """All-gather of per-rank attention outputs in KV-head-sharded mode.

    `gather(local)` takes this rank's [B, Hq/n, D] output and returns the full
    [B, Hq, D] in head order, using all_gather_into_tensor into a
    preallocated buffer (rank-major [n, B, Hq/n, D], then a local transpose)."""

    def __init__(self, world: int, group: Optional["torch.distributed.ProcessGroup"] = None):
        self.world = int(world)
        self.group = group
        self._buf: Optional[torch.Tensor] = None

    def gather(self, local: torch.Tensor) -> torch.Tensor:
        import torch.distributed as dist

        local = local.contiguous()
        B, hq_local, D = local.shape
        shape = (self.world * B, hq_local, D)  # rank-major
        if self._buf is None or tuple(self._buf.shape) != shape or self._buf.dtype != local.dtype \
                or self._buf.device != local.device:
            self._buf = torch.empty(shape, dtype=local.dtype, device=local.device)
        dist.all_gather_into_tensor(self._buf, local, group=self.group)
        return self._buf.view(self.world, B, hq_local, D).permute(1, 0, 2, 3).reshape(B, self.world * hq_local, D)
