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


def hybrid_grid(num_kv_heads: int, batch: int, world: int, min_heads: int = 4):
    """(head_parts, batch_parts) for `world` ranks: split kv heads while each
    shard keeps at least `min_heads` of them (a K slice of fewer heads per
    block streams less efficiently), then split the batch."""
    hp = 1
    while hp * 2 <= world and num_kv_heads % (hp * 2) == 0 and num_kv_heads // (hp * 2) >= min_heads:
        hp *= 2
    dp = world // hp
    if hp * dp != world or batch % dp != 0:
        raise ValueError(f"cannot split {num_kv_heads} kv heads x {batch} sequences over {world} ranks")
    return hp, dp


def hybrid_coords(rank: int, hp: int):
    """(head part, batch part) of `rank`: ranks of one batch part are adjacent."""
    return rank % hp, rank // hp


def assemble_hybrid(parts, hp: int, dp: int):
    """Rank-ordered outputs [B/dp, Hq/hp, D] -> [B, Hq, D]."""
    import torch
    rows = [torch.cat([parts[d * hp + h] for h in range(hp)], dim=1) for d in range(dp)]
    return torch.cat(rows, dim=0)


def all_gather_hybrid(out_shard, hp: int, dp: int, group=None, gathered=None, result=None):
    """All-gather of every rank's [B/dp, Hq/hp, D] output, reassembled to
    [B, Hq, D]: one NCCL all_gather_into_tensor into `gathered` (rank-major
    [dp, hp, B/dp, Hq/hp, D]) and one reordering copy into `result`. Both
    buffers are allocated when not given (pass them to keep a step
    allocation-free, e.g. inside a CUDA graph)."""
    import torch
    import torch.distributed as dist
    b, h, d = out_shard.shape
    if gathered is None:
        gathered = torch.empty((dp, hp, b, h, d), dtype=out_shard.dtype, device=out_shard.device)
    if result is None:
        result = torch.empty((dp * b, hp * h, d), dtype=out_shard.dtype, device=out_shard.device)
    dist.all_gather_into_tensor(gathered.view(-1), out_shard.contiguous().view(-1), group=group)
    result.view(dp, b, hp, h, d).copy_(gathered.permute(0, 2, 1, 3, 4))
    return result


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


def all_gather_heads(out_shard, group=None, gathered=None, result=None):
    """torch.distributed all-gather of a rank's [B, Hq/N, D] output, then the
    head reassembly to [B, Hq, D]. Works with NCCL (CUDA tensors) and gloo
    (CPU tensors)."""
    import torch.distributed as dist
    return all_gather_hybrid(out_shard, dist.get_world_size(group), 1, group, gathered, result)
