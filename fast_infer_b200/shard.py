"""Partitioning of the attention path across the GPUs of one node.

Attention needs no exchange between GPUs: each query head reads exactly one KV
head (GQA, h -> h // (Hq/Hkv)) and each sequence its own pages. So the path shards
with no collective on the data path, one process per GPU:

* by KV head — rank r of N owns KV heads [r*Hkv/N, (r+1)*Hkv/N) and the query heads
  that read them (contiguous, since the group of KV head j is [j*G, (j+1)*G)); each
  rank keeps a KVCache with Hkv/N heads and the full (replicated) block table;
* by sequence — rank r owns a contiguous slice of the batch with all heads.

The only collective is ``gather_heads``: where a caller needs the attention output
whole (the O projection of a tensor-parallel-free layer), the per-rank
[tokens, heads_r*D] outputs are all-gathered (NCCL over NVLink on B200; gloo in the
CPU tests) and reassembled in head order.
"""

from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class HeadShard:
    rank: int
    world: int
    kv_start: int
    kv_end: int
    q_start: int
    q_end: int

    @property
    def num_kv_heads(self) -> int:
        return self.kv_end - self.kv_start

    @property
    def num_q_heads(self) -> int:
        return self.q_end - self.q_start


def head_shard(rank: int, world: int, num_q_heads: int, num_kv_heads: int) -> HeadShard:
    """KV-head partition of rank ``rank`` of ``world`` (KV heads must divide evenly)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} / world {world}")
    if num_kv_heads % world != 0:
        raise ValueError(f"{num_kv_heads} KV heads do not split over {world} ranks")
    if num_q_heads % num_kv_heads != 0:
        raise ValueError("num_q_heads must be a multiple of num_kv_heads")
    per = num_kv_heads // world
    g = num_q_heads // num_kv_heads
    kv0 = rank * per
    return HeadShard(rank, world, kv0, kv0 + per, kv0 * g, (kv0 + per) * g)


def seq_range(rank: int, world: int, batch: int) -> tuple[int, int]:
    """Contiguous batch slice of a rank (sizes differ by at most one)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} / world {world}")
    base, extra = divmod(batch, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def shard_heads(x, shard: HeadShard, kv: bool, dim: int = 1):
    """Slice a tensor's head dimension to this rank's query (kv=False) or KV heads."""
    lo, hi = (shard.kv_start, shard.kv_end) if kv else (shard.q_start, shard.q_end)
    return x.narrow(dim, lo, hi - lo)


def gather_heads(local, group=None, head_dim_axis: int = -1):
    """All-gather per-rank attention outputs along the flattened head axis.

    ``local``: [..., heads_r * D] of this rank (equal shapes on every rank). Returns
    [..., world * heads_r * D] with rank r's block at position r, i.e. the heads in
    their original order. Uses torch.distributed (NCCL on GPUs, gloo on CPU).
    """
    import torch
    import torch.distributed as dist
    world = dist.get_world_size(group)
    if world == 1:
        return local
    local = local.contiguous()
    parts = [torch.empty_like(local) for _ in range(world)]
    dist.all_gather(parts, local, group=group)
    return torch.cat(parts, dim=head_dim_axis)
