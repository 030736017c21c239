"""KV-head sharding of the paged-decode path across GPUs.

Rank r of N owns kv heads [r*Hkv/N, (r+1)*Hkv/N) and the query heads that
read them ([r*Hq/N, (r+1)*Hq/N), since query head h reads kv head h / G).
Host bookkeeping (allocator, tables, copy-on-write, swap) is replicated: every
rank runs the same operations and gets the same block ids, so the same block
tables apply to every shard; only the bytes per block differ (the shard's
heads). Decode needs no exchange. When a consumer needs all heads on one GPU,
the per-rank outputs [B, Hq/N, D] are all-gathered (NCCL over NVLink on
GPUs, gloo in the CPU tests) and interleaved back to [B, Hq, D].
"""
from __future__ import annotations

import numpy as np


def head_range(num_kv_heads: int, world: int, rank: int):
    if num_kv_heads % world != 0:
        raise ValueError(f"{num_kv_heads} kv heads do not split over {world} ranks")
    per = num_kv_heads // world
    return rank * per, (rank + 1) * per


def shard_pool(pool: np.ndarray, w, world: int, rank: int) -> np.ndarray:
    """The shard of a host pool image (uint8 [num_blocks*stride]) holding
    this rank's kv heads, laid out as a pool of num_kv_heads/world heads."""
    h0, h1 = head_range(w.num_kv_heads, world, rank)
    full = pool.reshape(w.num_blocks, w.block_stride)[:, : w.block_bytes]
    row = w.head_dim * w.elem
    # [block][layer][K|V][token][head][head_dim bytes]
    v = full.reshape(w.num_blocks, w.num_layers, 2, w.tokens_per_block, w.num_kv_heads, row)
    part = np.ascontiguousarray(v[:, :, :, :, h0:h1, :]).reshape(w.num_blocks, -1)
    shard_bytes = part.shape[1]
    stride = (max(shard_bytes, 1) + 255) // 256 * 256
    out = np.zeros((w.num_blocks, stride), dtype=np.uint8)
    out[:, :shard_bytes] = part
    return out.reshape(-1)


def shard_query(q: np.ndarray, num_kv_heads: int, world: int, rank: int) -> np.ndarray:
    hq = q.shape[1]
    per = hq // world
    return np.ascontiguousarray(q[:, rank * per:(rank + 1) * per])


def shard_workload(w, world: int):
    """The same workload seen by one shard (kv and query heads divided)."""
    import copy
    s = copy.copy(w)
    s.num_kv_heads = w.num_kv_heads // world
    s.num_query_heads = w.num_query_heads // world
    return s


def assemble(gathered, axis: int = 1):
    """Per-rank outputs [B, Hq/N, D] (rank order) -> [B, Hq, D]."""
    return np.concatenate(list(gathered), axis=axis)


def all_gather_heads(out_shard, group=None):
    """torch.distributed all-gather of a rank's [B, Hq/N, D] output, then the
    head reassembly. Works with NCCL (CUDA tensors) and gloo (CPU tensors)."""
    import torch
    import torch.distributed as dist
    world = dist.get_world_size(group)
    parts = [torch.empty_like(out_shard) for _ in range(world)]
    dist.all_gather(parts, out_shard.contiguous(), group=group)
    return torch.cat(parts, dim=1)
