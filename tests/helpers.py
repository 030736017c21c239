"""Test helpers: reference-style cache fixtures and a GPU runner.

`pattern` and the scattered-table fixture restate the reference test suite's
helpers (phhuang191129/QwenVL-Paged tests/PagedAttention.test.cpp:80-92 and
:209-241) so the known-answer tests read like the reference's own.
"""
from __future__ import annotations

import math

import numpy as np

import workloads as W


def pattern(layer: int, stream: int, token: int, head: int, dim: int) -> float:
    """FNV-1a style mix of the coordinates mapped into [-1, 1)
    (tests/PagedAttention.test.cpp:80-92)."""
    mixed = 2166136261
    for part in (layer, stream, token, head, dim):
        mixed = ((mixed ^ part) * 16777619) & 0xFFFFFFFF
    return np.float32(mixed % 2000) / np.float32(1000.0) - np.float32(1.0)


class HostCache:
    """A flat host image of a block pool plus per-sequence tables."""

    def __init__(self, *, tokens_per_block, num_layers, num_kv_heads, head_dim, dtype="f32", num_blocks=8):
        self.T, self.L, self.H, self.D = tokens_per_block, num_layers, num_kv_heads, head_dim
        self.dtype = dtype
        self.elem = 4 if dtype == "f32" else 2
        self.num_blocks = num_blocks
        self.block_bytes = self.T * self.L * self.H * self.D * self.elem * 2
        self.stride = (max(self.block_bytes, 1) + 255) // 256 * 256
        self.pool = np.zeros(num_blocks * self.stride, dtype=np.uint8)

    def offset(self, layer, stream, t, h):
        """KVBlockLayout::element_offset (src/CacheLayout.cpp:25-38)."""
        head = self.D
        token = self.H * head
        strm = self.T * token
        return layer * 2 * strm + stream * strm + t * token + h * head

    def write(self, block, layer, stream, t, h, vec):
        vec = np.asarray(vec, dtype=np.float32)
        if self.dtype == "bf16":
            raw = W.f32_to_bf16_bits(vec).view(np.uint8)
        else:
            raw = vec.view(np.uint8)
        start = block * self.stride + self.offset(layer, stream, t, h) * self.elem
        self.pool[start:start + raw.size] = raw

    def workload(self, *, hq, scale, context_lens, tables, layer=0):
        ctx = np.asarray(context_lens, dtype=np.int32)
        tab = np.asarray(tables, dtype=np.int32)
        if tab.ndim == 1:
            tab = tab[None, :]
        return W.DecodeWorkload("fixture", self.T, self.L, self.H, self.D, self.dtype, hq, scale, ctx, tab,
                                self.num_blocks, 0, layer=layer)


def scattered_ids(num_blocks: int, blocks: int):
    """Frames the reference allocator hands a sequence that alternates with a
    spacer sequence: the free list is LIFO over 0..N-1, so the sequence gets
    N-1, N-3, N-5, ... (tests/PagedAttention.test.cpp:209-218, 222-223)."""
    return [num_blocks - 1 - 2 * i for i in range(blocks)]


def gpu_decode(w, pool: np.ndarray, q: np.ndarray, *, split_tokens=0, context_lens=None, tables=None,
               max_context_len=None, out_init=None, pool_dev=None):
    """Runs qvp_decode on cuda:0. Returns (status, out float32, error word, plan)."""
    import torch

    import qvp

    dev = torch.device("cuda", 0)
    ctx = np.ascontiguousarray(w.context_lens if context_lens is None else context_lens, dtype=np.int32)
    tab = np.ascontiguousarray(w.tables if tables is None else tables, dtype=np.int32)
    if pool_dev is None:
        pool_dev = torch.from_numpy(np.ascontiguousarray(pool)).to(dev)
    qt = torch.from_numpy(np.ascontiguousarray(q).view(np.int16 if w.dtype == "bf16" else np.float32)).to(dev)
    if w.dtype == "bf16":
        qt = qt.view(torch.bfloat16)
    out_dtype = torch.bfloat16 if w.dtype == "bf16" else torch.float32
    out = torch.zeros((len(ctx), w.num_query_heads, w.head_dim), dtype=out_dtype, device=dev)
    if out_init is not None:
        out.fill_(out_init)
    ctx_d = torch.from_numpy(ctx).to(dev)
    tab_d = torch.from_numpy(tab).to(dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    shape = qvp.make_shape(w.tokens_per_block, w.num_layers, w.num_kv_heads, w.head_dim, w.elem)
    mcl = int(max_context_len if max_context_len is not None else max(int(ctx.max()), 1))
    args = qvp.decode_args(pool=pool_dev.data_ptr(), block_stride=w.block_stride, num_blocks=w.num_blocks,
                           shape=shape, dtype=qvp.DTYPE_F32 if w.dtype == "f32" else qvp.DTYPE_BF16,
                           layer=w.layer, num_query_heads=w.num_query_heads, scale=w.scale, batch=len(ctx),
                           max_blocks_per_seq=tab.shape[1], max_context_len=mcl,
                           block_tables=tab_d.data_ptr(), context_lens=ctx_d.data_ptr(), query=qt.data_ptr(),
                           out=out.data_ptr(), split_tokens=split_tokens, error_word=err.data_ptr())
    plan = None
    ws = None
    try:
        plan = qvp.decode_plan(args)
        if plan["workspace_bytes"]:
            ws = torch.empty(plan["workspace_bytes"], dtype=torch.uint8, device=dev)
            args.workspace = ws.data_ptr()
            args.workspace_bytes = plan["workspace_bytes"]
    except qvp.QvpError:
        pass
    status = qvp.decode(args, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    return status, out.float().cpu().numpy(), int(err.item()), plan


def max_rel_err(got: np.ndarray, ref: np.ndarray) -> float:
    """max |got - ref| / max |ref| (the 1e-5 relative criterion for fp32)."""
    scale = float(np.max(np.abs(ref))) or 1.0
    return float(np.max(np.abs(got - ref))) / scale


def bf16_f32(q: np.ndarray) -> np.ndarray:
    return W.bf16_bits_to_f32(q)


def mean_ctx(ctx) -> float:
    return float(np.mean(ctx)) if len(ctx) else math.nan


class NativeCases:
    """A native test library built on tests/native/harness.h: `<prefix>_list`
    names its cases, `<prefix>_run(name)` runs one (0 = passed, failure text
    otherwise)."""

    def __init__(self, path: str, prefix: str):
        self.path, self.prefix = path, prefix

    def _lib(self):
        import ctypes as C
        return C.CDLL(self.path)

    def names(self):
        import ctypes as C
        import os
        if not os.path.exists(self.path):
            return []
        buf = C.create_string_buffer(1 << 16)
        getattr(self._lib(), f"{self.prefix}_list")(buf, len(buf))
        return [n for n in buf.value.decode().splitlines() if n]

    def run(self, name: str):
        """(return code, message) of one case."""
        import ctypes as C
        msg = C.create_string_buffer(4096)
        rc = getattr(self._lib(), f"{self.prefix}_run")(name.encode(), msg, len(msg))
        return rc, msg.value.decode()


def device_bytes(ptr: int, nbytes: int, dev):
    """A uint8 torch view of `nbytes` of device memory at `ptr` (memory libqvp owns)."""
    import torch

    class _Raw:
        __cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False), "version": 3,
                                    "strides": None}

    return torch.as_tensor(_Raw(), device=dev)
