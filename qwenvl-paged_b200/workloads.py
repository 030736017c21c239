"""Seeded synthetic decode workloads with the shapes of the benchmark configs.

No public dataset is involved: every config is a shape plus a seed. K, V and
Q are i.i.d. N(0, 1); context lengths and the scattered block tables come
from numpy's PCG64 generator with a committed seed, so the GPU run, the CPU
oracle and the reference see the same bytes.

Configs (the block layout is [layer][K|V][token][kv_head][head_dim]):
  cfg1  4 sequences, ctx {37,128,255,512}, 16-token blocks, 8 query / 2 kv
        heads, head_dim 64, fp32, tables a permutation of a 256-block pool.
  cfg2  Qwen2-VL-7B-shaped: 64 sequences, ctx ~ U[512, 8192], 28 / 4 heads,
        head_dim 128, bf16, pool 1.25x the blocks used.
  cfg3  copy-on-write parallel sampling over cfg2 shapes (see cow.py).
  cfg4  Qwen2-VL-72B-shaped: 32 sequences of 32768 tokens, 64 / 8 heads,
        head_dim 128, bf16, sharded by kv head over 1/2/4/8 GPUs.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even float32 -> bfloat16 bit patterns (uint16)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return r


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


@dataclass
class DecodeWorkload:
    name: str
    tokens_per_block: int
    num_layers: int
    num_kv_heads: int
    head_dim: int
    dtype: str                  # "f32" or "bf16"
    num_query_heads: int
    scale: float
    context_lens: np.ndarray    # int32 [B]
    tables: np.ndarray          # int32 [B, pitch], -1 past each context
    num_blocks: int
    seed: int
    layer: int = 0
    meta: dict = field(default_factory=dict)

    @property
    def batch(self) -> int:
        return int(self.context_lens.shape[0])

    @property
    def elem(self) -> int:
        return 4 if self.dtype == "f32" else 2

    @property
    def pitch(self) -> int:
        return int(self.tables.shape[1])

    @property
    def block_bytes(self) -> int:
        return self.tokens_per_block * self.num_layers * self.num_kv_heads * self.head_dim * self.elem * 2

    @property
    def block_stride(self) -> int:
        return (max(self.block_bytes, 1) + 255) // 256 * 256

    @property
    def max_context_len(self) -> int:
        return int(self.context_lens.max())

    def kv_bytes(self) -> int:
        """K and V bytes one decode step must read (each once per step)."""
        return int(self.context_lens.astype(np.int64).sum()) * self.num_kv_heads * self.head_dim * self.elem * 2

    def algorithmic_bytes(self) -> int:
        """KV + Q + out + the block-table entries used."""
        qo = 2 * self.batch * self.num_query_heads * self.head_dim * self.elem
        tbl = int(np.ceil(self.context_lens / self.tokens_per_block).sum()) * 4
        return self.kv_bytes() + qo + tbl

    def flops(self) -> int:
        return 4 * self.num_query_heads * self.head_dim * int(self.context_lens.astype(np.int64).sum())


def scattered_tables(rng: np.random.Generator, context_lens: np.ndarray, tokens_per_block: int,
                     num_blocks: int) -> np.ndarray:
    """Block ids drawn in order from a seeded permutation of the pool."""
    need = [int(math.ceil(c / tokens_per_block)) for c in context_lens]
    pitch = max(need)
    assert sum(need) <= num_blocks, "pool too small"
    perm = rng.permutation(num_blocks).astype(np.int32)
    tables = np.full((len(need), pitch), -1, dtype=np.int32)
    pos = 0
    for b, n in enumerate(need):
        tables[b, :n] = perm[pos:pos + n]
        pos += n
    return tables


def cfg1(seed: int = 1) -> DecodeWorkload:
    rng = np.random.default_rng(seed)
    ctx = np.array([37, 128, 255, 512], dtype=np.int32)
    tables = scattered_tables(rng, ctx, 16, 256)
    return DecodeWorkload("cfg1-cpu-reference-decode", 16, 1, 2, 64, "f32", 8, 1.0 / 8.0, ctx, tables, 256, seed)


def cfg2(seed: int = 2, batch: int = 64, lo: int = 512, hi: int = 8192) -> DecodeWorkload:
    rng = np.random.default_rng(seed)
    ctx = rng.integers(lo, hi + 1, size=batch).astype(np.int32)
    used = int(np.ceil(ctx / 16).sum())
    num_blocks = int(math.ceil(1.25 * used))
    tables = scattered_tables(rng, ctx, 16, num_blocks)
    return DecodeWorkload("cfg2-qwen2vl-7b-decode", 16, 1, 4, 128, "bf16", 28, 1.0 / math.sqrt(128), ctx, tables,
                          num_blocks, seed)


def cfg2_shard(head_parts: int = 1, seed: int = 2) -> DecodeWorkload:
    """What one GPU holds when the 7B-shaped decode is split by kv head over
    `head_parts` GPUs at constant bytes per GPU: a batch of 64*head_parts
    sequences (ctx ~ U[512, 8192], seeded), of which this GPU owns
    4/head_parts kv heads and their 28/head_parts query heads. head_parts = 1
    is cfg2 itself."""
    if head_parts not in (1, 2, 4):
        raise ValueError(f"cfg2 has 4 kv heads; cannot split them {head_parts} ways")
    w = cfg2(seed=seed, batch=64 * head_parts)
    if head_parts > 1:
        w.num_kv_heads //= head_parts
        w.num_query_heads //= head_parts
        w.name = f"cfg2-qwen2vl-7b-decode-kvshard{head_parts}"
    w.meta = {"head_parts": head_parts}
    return w


def cfg4(seed: int = 4, batch: int = 32, ctx_len: int = 32768, shards: int = 1) -> DecodeWorkload:
    """One kv-head shard of the 72B-shaped config (8 // shards kv heads)."""
    assert 8 % shards == 0
    rng = np.random.default_rng(seed)
    ctx = np.full(batch, ctx_len, dtype=np.int32)
    used = int(np.ceil(ctx / 16).sum())
    tables = scattered_tables(rng, ctx, 16, used)
    # 80% of each context tagged as image/video spans: metadata only, the
    # values stay N(0, 1) and the kernel never reads the tags.
    span_start = rng.integers(0, ctx_len - int(0.8 * ctx_len) + 1, size=batch)
    w = DecodeWorkload("cfg4-qwen2vl-72b-long-decode", 16, 1, 8 // shards, 128, "bf16", 64 // shards,
                       1.0 / math.sqrt(128), ctx, tables, used, seed)
    w.meta = {"shards": shards, "multimodal_spans": [(int(s), int(0.8 * ctx_len)) for s in span_start]}
    return w


def small(seed: int, *, batch: int, ctx_lo: int, ctx_hi: int, hq: int, hkv: int, head_dim: int, dtype: str,
          tokens_per_block: int = 16, num_layers: int = 1, layer: int = 0, pool_factor: float = 1.5,
          scale: float | None = None) -> DecodeWorkload:
    """A reduced workload for parity tests (same generator as the configs)."""
    rng = np.random.default_rng(seed)
    ctx = rng.integers(ctx_lo, ctx_hi + 1, size=batch).astype(np.int32)
    used = int(np.ceil(ctx / tokens_per_block).sum())
    num_blocks = max(int(math.ceil(pool_factor * used)), used)
    tables = scattered_tables(rng, ctx, tokens_per_block, num_blocks)
    return DecodeWorkload(f"small-{seed}", tokens_per_block, num_layers, hkv, head_dim, dtype, hq,
                          scale if scale is not None else 1.0 / math.sqrt(head_dim), ctx, tables, num_blocks, seed,
                          layer=layer)


def with_contexts(w: DecodeWorkload, context_lens) -> DecodeWorkload:
    """The same workload with new context lengths and tables re-drawn for them."""
    rng = np.random.default_rng(w.seed + 77)
    ctx = np.asarray(context_lens, dtype=np.int32)
    used = int(np.ceil(ctx / w.tokens_per_block).sum())
    num_blocks = max(w.num_blocks, used)
    tables = scattered_tables(rng, ctx, w.tokens_per_block, num_blocks)
    return DecodeWorkload(w.name, w.tokens_per_block, w.num_layers, w.num_kv_heads, w.head_dim, w.dtype,
                          w.num_query_heads, w.scale, ctx, tables, num_blocks, w.seed, layer=w.layer)


def host_inputs(w: DecodeWorkload, seed_offset: int = 1000):
    """(pool bytes as uint8 [num_blocks*stride], query array) in the workload dtype.

    bf16 values are stored as uint16 bit patterns. Padding bytes past each
    block's payload are zero.
    """
    rng = np.random.default_rng(w.seed + seed_offset)
    n_el = w.block_bytes // w.elem
    vals = rng.standard_normal((w.num_blocks, n_el), dtype=np.float32)
    q = rng.standard_normal((w.batch, w.num_query_heads, w.head_dim), dtype=np.float32)
    if w.dtype == "bf16":
        vals = f32_to_bf16_bits(vals)
        q = f32_to_bf16_bits(q)
    pool = np.zeros((w.num_blocks, w.block_stride), dtype=np.uint8)
    pool[:, :w.block_bytes] = vals.view(np.uint8).reshape(w.num_blocks, w.block_bytes)
    return pool.reshape(-1), q
