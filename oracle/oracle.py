"""TEST INFRASTRUCTURE ONLY - Python handles on the CPU oracle.

Loaded only by tests/, __graft_entry__.smoke() and bench.py (as the checker
and as the timed CPU baseline). Two back ends:

  * ``port``      - oracle/lib/liboracle.so, the plain-C restatement of
                    paged_attention_decode<T> (paged_decode_oracle.c).
  * ``reference`` - oracle/_ref/libqvp_ref.so, the reference's own sources
                    (phhuang191129/QwenVL-Paged src/*.cpp and
                    include/qwenvl_paged/PagedAttention.h) compiled by
                    oracle/Makefile. Present wherever it was built.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
PORT_PATH = os.path.join(_HERE, "lib", "liboracle.so")
REF_PATH = os.path.join(_HERE, "_ref", "libqvp_ref.so")


class Shape(C.Structure):
    _fields_ = [("tokens_per_block", C.c_uint32), ("num_layers", C.c_uint32), ("num_kv_heads", C.c_uint32),
                ("head_dim", C.c_uint32), ("bytes_per_element", C.c_uint32)]


_port = None
_ref = None


def port_lib() -> C.CDLL:
    global _port
    if _port is None:
        if not os.path.exists(PORT_PATH):
            raise ImportError(f"{PORT_PATH} missing; run `make -C oracle`")
        lib = C.CDLL(PORT_PATH)
        vp, u32 = C.c_void_p, C.c_uint32
        lib.oracle_paged_decode.restype = C.c_int
        lib.oracle_paged_decode.argtypes = [vp, C.c_size_t, u32, C.POINTER(Shape), C.c_int, u32, u32, C.c_float,
                                            vp, u32, u32, vp, vp]
        lib.oracle_paged_decode_batch.restype = C.c_int
        lib.oracle_paged_decode_batch.argtypes = [vp, C.c_size_t, u32, C.POINTER(Shape), C.c_int, u32, u32,
                                                  C.c_float, u32, u32, vp, vp, vp, vp, vp, C.c_int]
        lib.oracle_copy_blocks.restype = None
        lib.oracle_copy_blocks.argtypes = [vp, C.c_size_t, u32, C.c_size_t, vp, u32]
        _port = lib
    return _port


def ref_available() -> bool:
    return os.path.exists(REF_PATH)


def ref_lib() -> C.CDLL:
    global _ref
    if _ref is None:
        if not os.path.exists(REF_PATH):
            raise ImportError(f"{REF_PATH} missing; build it with `make -C oracle REF=<reference checkout>`")
        lib = C.CDLL(REF_PATH)
        vp, u32 = C.c_void_p, C.c_uint32
        lib.ref_pool_create.restype = vp
        lib.ref_pool_create.argtypes = [C.POINTER(Shape), u32, vp, C.c_size_t]
        lib.ref_pool_destroy.restype = None
        lib.ref_pool_destroy.argtypes = [vp]
        lib.ref_tables_create.restype = vp
        lib.ref_tables_create.argtypes = [vp, u32, u32, vp, vp]
        lib.ref_tables_destroy.restype = None
        lib.ref_tables_destroy.argtypes = [vp]
        lib.ref_decode_bound.restype = C.c_int
        lib.ref_decode_bound.argtypes = [vp, vp, C.c_int, u32, u32, C.c_float, u32, vp, vp, vp, vp, C.c_int]
        lib.ref_decode_batch.restype = C.c_int
        lib.ref_decode_batch.argtypes = [vp, C.c_int, u32, u32, C.c_float, u32, u32, vp, vp, vp, vp, vp, C.c_int]
        if hasattr(lib, "ref_replay"):
            lib.ref_replay.restype = C.c_int
            lib.ref_replay.argtypes = [C.c_char_p, C.c_char_p, C.c_size_t]
        _ref = lib
    return _ref


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


def _shape(w) -> Shape:
    return Shape(w.tokens_per_block, w.num_layers, w.num_kv_heads, w.head_dim, w.elem)


def port_decode(w, pool: np.ndarray, q: np.ndarray, threads: int = 1, context_lens=None, tables=None):
    """Oracle outputs (float32 [B, Hq, D]) and per-sequence status."""
    ctx = np.ascontiguousarray(w.context_lens if context_lens is None else context_lens, dtype=np.int32)
    tab = np.ascontiguousarray(w.tables if tables is None else tables, dtype=np.int32)
    pool = np.ascontiguousarray(pool)
    q = np.ascontiguousarray(q)
    out = np.zeros((len(ctx), w.num_query_heads, w.head_dim), dtype=np.float32)
    status = np.zeros(len(ctx), dtype=np.int32)
    sh = _shape(w)
    port_lib().oracle_paged_decode_batch(_ptr(pool), w.block_stride, w.num_blocks, C.byref(sh),
                                         0 if w.dtype == "f32" else 1, w.layer, w.num_query_heads, w.scale,
                                         len(ctx), tab.shape[1], _ptr(tab), _ptr(ctx), _ptr(q), _ptr(out),
                                         _ptr(status), threads)
    return out, status


class RefDecoder:
    """The reference's paged_attention_decode<T> over a copy of the pool."""

    def __init__(self, w, pool: np.ndarray):
        self.w = w
        self.lib = ref_lib()
        self.sh = _shape(w)
        pool = np.ascontiguousarray(pool)
        self.h = self.lib.ref_pool_create(C.byref(self.sh), w.num_blocks, _ptr(pool), w.block_stride)
        self.tables_h = None

    def bind(self, context_lens=None, tables=None):
        w = self.w
        self.ctx = np.ascontiguousarray(w.context_lens if context_lens is None else context_lens, dtype=np.int32)
        self.tab = np.ascontiguousarray(w.tables if tables is None else tables, dtype=np.int32)
        if self.tables_h is not None:
            self.lib.ref_tables_destroy(self.tables_h)
        self.tables_h = self.lib.ref_tables_create(self.h, len(self.ctx), self.tab.shape[1], _ptr(self.tab),
                                                   _ptr(self.ctx))

    def decode(self, q: np.ndarray, threads: int = 1):
        """Outputs in the workload dtype (bf16 as uint16 bits) and status."""
        w = self.w
        if self.tables_h is None:
            self.bind()
        q = np.ascontiguousarray(q)
        out = np.zeros((len(self.ctx), w.num_query_heads, w.head_dim),
                       dtype=np.float32 if w.dtype == "f32" else np.uint16)
        status = np.zeros(len(self.ctx), dtype=np.int32)
        self.lib.ref_decode_bound(self.h, self.tables_h, 0 if w.dtype == "f32" else 1, w.layer,
                                  w.num_query_heads, w.scale, len(self.ctx), _ptr(self.ctx), _ptr(q), _ptr(out),
                                  _ptr(status), threads)
        return out, status

    def close(self):
        if self.tables_h is not None:
            self.lib.ref_tables_destroy(self.tables_h)
            self.tables_h = None
        if self.h:
            self.lib.ref_pool_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def port_copy_blocks(pool: np.ndarray, block_stride: int, num_blocks: int, nbytes: int, pairs: np.ndarray):
    pairs = np.ascontiguousarray(pairs, dtype=np.int32)
    port_lib().oracle_copy_blocks(_ptr(pool), block_stride, num_blocks, nbytes, _ptr(pairs), len(pairs) // 2)


def prefill_pairs(w, query_lens):
    """(sequence, token) pairs of a prefill and, per pair, the context length
    the reference would decode with: position + 1 (PagedAttention.h:43-44)."""
    seq, tok, ctx = [], [], []
    for b, (c, ql) in enumerate(zip(w.context_lens, query_lens)):
        for t in range(int(ql)):
            seq.append(b)
            tok.append(t)
            ctx.append(int(c) - int(ql) + t + 1)
    return np.array(seq, dtype=np.int64), np.array(tok, dtype=np.int64), np.array(ctx, dtype=np.int32)


def port_prefill(w, pool, q, query_lens, threads=1):
    """Prefill as the reference defines it: the decode at every query
    position. q is [B, max_qlen, Hq, D]; returns float32 [B, max_qlen, Hq, D]
    (rows past each query length stay zero) and the per-pair status."""
    seq, tok, ctx = prefill_pairs(w, query_lens)
    out = np.zeros((w.batch,) + tuple(q.shape[1:]), dtype=np.float32)
    if len(seq) == 0:
        return out, np.zeros(0, dtype=np.int32)
    tables = np.ascontiguousarray(w.tables[seq])
    qq = np.ascontiguousarray(q[seq, tok])
    o, status = port_decode(w, pool, qq, threads=threads, context_lens=ctx, tables=tables)
    out[seq, tok] = o
    return out, status


# ---- compressed swap slots ----------------------------------------------------
# The reference stores a swapped block's bytes verbatim
# (src/SwapBackend.cpp:10-39); a compressed slot must give back exactly those
# bytes. The slot format (header, 4-bit high-byte codes over a 15-entry
# dictionary, raw low bytes, u32 escapes) is restated here in numpy so the
# tests can check the device coder byte for byte, not only by round trip.

SLOT_CODED = 0x31505651  # "QVP1"
SLOT_RAW = 0x30505651    # "QVP0"


def swap_slot_bytes(block_bytes: int) -> int:
    return (block_bytes + 16 + 15) // 16 * 16


def port_compress_block(block: np.ndarray) -> tuple[np.ndarray, set]:
    """Codes one block (uint8 array). Returns (slot bytes of length
    swap_slot_bytes, set of escape words). The escape list's order is free in
    the format (the device coder appends them as they are found); this one
    writes them in index order and also returns them as a set."""
    nb = block.size
    slot = np.zeros(swap_slot_bytes(nb), dtype=np.uint8)
    n = nb // 2
    codable = nb % 32 == 0 and n < (1 << 24)
    escapes: set = set()
    if codable:
        vals = block.view(np.uint16)
        hi = (vals >> 8).astype(np.int64)
        lo = (vals & 0xFF).astype(np.uint8)
        hist = np.bincount(hi, minlength=256)
        # rank by count descending, ties to the smaller byte
        order = sorted(range(256), key=lambda u: (-hist[u], u))
        code_of = np.full(256, 15, dtype=np.uint8)
        dictionary = np.zeros(16, dtype=np.uint8)
        for r, u in enumerate(order[:15]):
            if hist[u] > 0:
                code_of[u] = r
                dictionary[r] = u
        codes = code_of[hi]
        esc_idx = np.nonzero(codes == 15)[0]
        used = 32 + n * 3 // 2 + 4 * len(esc_idx)
        if used < 16 + nb:
            slot[:16] = np.array([SLOT_CODED, len(esc_idx), used, 0], dtype=np.uint32).view(np.uint8)
            slot[16:32] = dictionary
            slot[32:32 + n // 2] = (codes[0::2] | (codes[1::2] << 4)).astype(np.uint8)
            slot[32 + n // 2:32 + n * 3 // 2] = lo
            words = (esc_idx.astype(np.uint32) << 8) | hi[esc_idx].astype(np.uint32)
            e0 = 32 + n * 3 // 2
            slot[e0:e0 + 4 * len(words)] = words.view(np.uint8)
            return slot, {int(x) for x in words}
    slot[:16] = np.array([SLOT_RAW, 0, 16 + nb, 0], dtype=np.uint32).view(np.uint8)
    slot[16:16 + nb] = block
    return slot, escapes


def port_decompress_slot(slot: np.ndarray, block_bytes: int) -> np.ndarray:
    """The block a slot codes (uint8 array of block_bytes)."""
    head = slot[:16].view(np.uint32)
    if head[0] == SLOT_RAW:
        return slot[16:16 + block_bytes].copy()
    assert head[0] == SLOT_CODED, "not a swap slot"
    n = block_bytes // 2
    dictionary = slot[16:32]
    packed = slot[32:32 + n // 2]
    codes = np.empty(n, dtype=np.uint8)
    codes[0::2] = packed & 15
    codes[1::2] = packed >> 4
    hi = np.where(codes < 15, dictionary[np.minimum(codes, 14)], 0).astype(np.uint16)
    lo = slot[32 + n // 2:32 + n * 3 // 2].astype(np.uint16)
    out = (hi << 8) | lo
    esc = slot[32 + n * 3 // 2:32 + n * 3 // 2 + 4 * int(head[1])].view(np.uint32)
    out[esc >> 8] = ((esc & 0xFF).astype(np.uint16) << 8) | lo[esc >> 8]
    return out.view(np.uint8).copy()
