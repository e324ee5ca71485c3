"""Partition of the delta-attention layer-op over GPUs by kv-head.

Every (batch, kv-head) unit of the path is independent: selection, packing and the two-phase
attention of kv-head h read only K / V / timestamps / counts of h and write only the output
rows of its query heads h*G .. h*G+G-1 (modeling_llama.py:638,665 launch one program per
(batch, head); deltaFlashAttention.py:28-32 map a program to its head). So a sequence splits
over `world` GPUs with no collective on the data path: rank r runs kv-heads
[r*Hkv/world, (r+1)*Hkv/world) with their query heads. The only collective is the optional
gather of the output for verification, outside any timed region.
"""
from __future__ import annotations

import torch


def kv_head_range(num_kv_heads: int, world: int, rank: int):
    """[first, last) kv-heads of `rank`; the kv-heads must divide evenly over the ranks."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    if num_kv_heads % world:
        raise ValueError(f"{num_kv_heads} kv-heads do not divide over {world} ranks")
    per = num_kv_heads // world
    return rank * per, (rank + 1) * per


def shard_layer(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, world: int, rank: int):
    """Views of q [B, Hq, N, d] and k / v [B, Hkv, N, d] that `rank` processes (no copies)."""
    Hq, Hkv = q.shape[1], k.shape[1]
    if Hq % Hkv:
        raise ValueError("query heads must be a multiple of kv-heads")
    G = Hq // Hkv
    ka, kb = kv_head_range(Hkv, world, rank)
    return q[:, ka * G:kb * G], k[:, ka:kb], v[:, ka:kb]


def gather_heads(out_local: torch.Tensor, world: int, group=None) -> torch.Tensor:
    """All-gather every rank's output heads [B, Hq/world, N, d] into [B, Hq, N, d], in rank
    (= head) order, on every rank."""
    import torch.distributed as dist
    if world == 1:
        return out_local
    x = out_local.contiguous()
    parts = [torch.empty_like(x) for _ in range(world)]
    dist.all_gather(parts, x, group=group)
    return torch.cat(parts, dim=1)
