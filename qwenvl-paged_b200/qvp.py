"""ctypes binding of libqvp.so, the B200 paged-decode C ABI (include/qvp.h).

The library is built in-tree (``make -C qwenvl-paged_b200``) and loaded from
``qwenvl-paged_b200/lib/libqvp.so``. There is no fallback: importing this
module without the built library raises, so a GPU run can never silently use
anything but the CUDA kernels.

Device memory, streams and collectives in tests and benchmarks come from
PyTorch; this module only ever sees raw addresses (Python ints).
"""
from __future__ import annotations

import ctypes as C
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "lib", "libqvp.so")

OK = 0
ERR_INVALID = 1
ERR_UNMAPPED = 2
ERR_CUDA = 3
ERR_DEVICE = 4
ERR_NOMEM = 5
ERR_UNSUPPORTED = 6
ERR_WORKSPACE = 7

DTYPE_F32 = 0
DTYPE_BF16 = 1

# Device error bits a kernel ORs into the caller's error word.
DEVERR_BAD_BLOCK = 1
DEVERR_TIMEOUT = 2
DEVERR_BAD_CONTEXT = 4


class QvpError(RuntimeError):
    def __init__(self, status: int, what: str):
        super().__init__(f"{what}: status {status}: {last_error()}")
        self.status = status


class BlockShape(C.Structure):
    """Field for field the reference BlockShape (Block.h:46-57)."""

    _fields_ = [
        ("tokens_per_block", C.c_uint32),
        ("num_layers", C.c_uint32),
        ("num_kv_heads", C.c_uint32),
        ("head_dim", C.c_uint32),
        ("bytes_per_element", C.c_uint32),
    ]


class DecodeArgs(C.Structure):
    _fields_ = [
        ("pool", C.c_void_p),
        ("block_stride", C.c_size_t),
        ("num_blocks", C.c_uint32),
        ("shape", BlockShape),
        ("dtype", C.c_int32),
        ("layer", C.c_uint32),
        ("num_query_heads", C.c_uint32),
        ("scale", C.c_float),
        ("batch", C.c_uint32),
        ("max_blocks_per_seq", C.c_uint32),
        ("max_context_len", C.c_uint32),
        ("block_tables", C.c_void_p),
        ("context_lens", C.c_void_p),
        ("query", C.c_void_p),
        ("out", C.c_void_p),
        ("split_tokens", C.c_uint32),
        ("workspace", C.c_void_p),
        ("workspace_bytes", C.c_size_t),
        ("error_word", C.c_void_p),
    ]


class PrefillArgs(C.Structure):
    _fields_ = [
        ("pool", C.c_void_p),
        ("block_stride", C.c_size_t),
        ("num_blocks", C.c_uint32),
        ("shape", BlockShape),
        ("dtype", C.c_int32),
        ("layer", C.c_uint32),
        ("num_query_heads", C.c_uint32),
        ("scale", C.c_float),
        ("batch", C.c_uint32),
        ("max_blocks_per_seq", C.c_uint32),
        ("max_query_len", C.c_uint32),
        ("block_tables", C.c_void_p),
        ("context_lens", C.c_void_p),
        ("query_lens", C.c_void_p),
        ("query", C.c_void_p),
        ("out", C.c_void_p),
        ("error_word", C.c_void_p),
    ]


class Shard(C.Structure):
    _fields_ = [("shard", C.c_uint32), ("num_shards", C.c_uint32), ("device", C.c_int)]


class ShardDecodeArgs(C.Structure):
    _fields_ = [
        ("shard", Shard),
        ("decode", DecodeArgs),
        ("nccl_comm", C.c_void_p),
        ("gathered", C.c_void_p),
        ("out", C.c_void_p),
    ]


NCCL_ID_BYTES = 128
PEER_HANDLE_BYTES = 64


def _load() -> C.CDLL:
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"{LIB_PATH} is not built; run `make -C qwenvl-paged_b200` (or __graft_entry__.build())")
    lib = C.CDLL(LIB_PATH)
    vp, sz, u32, i32 = C.c_void_p, C.c_size_t, C.c_uint32, C.c_int32
    P = C.POINTER
    sig = {
        "qvp_block_bytes": (sz, [P(BlockShape)]),
        "qvp_block_stride": (sz, [P(BlockShape)]),
        "qvp_last_error": (C.c_char_p, []),
        "qvp_version": (C.c_char_p, []),
        "qvp_device_sm_count": (C.c_int, []),
        "qvp_pool_create": (C.c_int, [C.c_int, P(BlockShape), u32, P(vp)]),
        "qvp_pool_destroy": (C.c_int, [vp]),
        "qvp_pool_base": (vp, [vp]),
        "qvp_pool_stride": (sz, [vp]),
        "qvp_pool_num_blocks": (u32, [vp]),
        "qvp_pool_device": (C.c_int, [vp]),
        "qvp_pool_write": (C.c_int, [vp, u32, sz, vp, sz]),
        "qvp_pool_read": (C.c_int, [vp, u32, sz, vp, sz]),
        "qvp_decode_workspace_size": (C.c_int, [P(DecodeArgs), P(sz)]),
        "qvp_decode_plan": (C.c_int, [P(DecodeArgs), P(u32), P(u32), P(C.c_int)]),
        "qvp_decode": (C.c_int, [P(DecodeArgs), vp]),
        "qvp_decode_noalloc": (C.c_int, [P(DecodeArgs), vp]),
        "qvp_prefill": (C.c_int, [P(PrefillArgs), vp]),
        "qvp_copy_blocks": (C.c_int, [vp, sz, u32, sz, vp, u32, vp, vp]),
        "qvp_gather_blocks": (C.c_int, [vp, sz, u32, sz, vp, u32, vp, vp, vp]),
        "qvp_scatter_blocks": (C.c_int, [vp, sz, u32, sz, vp, u32, vp, vp, vp]),
        "qvp_swap_slot_bytes": (sz, [sz]),
        "qvp_fetch_host": (C.c_int, [vp, vp, sz, vp]),
        "qvp_compress_blocks": (C.c_int, [vp, sz, u32, sz, vp, vp, u32, vp, sz, vp, sz, u32, vp, vp, vp]),
        "qvp_decompress_blocks": (C.c_int, [vp, sz, u32, sz, vp, vp, u32, vp, sz, vp, sz, u32, vp, vp, vp]),
        "qvp_kv_append": (C.c_int, [vp, sz, u32, P(BlockShape), u32, u32, u32, vp, vp, vp, vp, vp, vp]),
        "qvp_shard_gather_bytes": (C.c_int, [P(ShardDecodeArgs), P(sz)]),
        "qvp_shard_decode": (C.c_int, [P(ShardDecodeArgs), vp]),
        "qvp_shard_reassemble": (C.c_int, [vp, vp, u32, u32, u32, u32, u32, vp]),
        "qvp_nccl_unique_id": (C.c_int, [vp, sz]),
        "qvp_nccl_comm_init": (C.c_int, [vp, sz, C.c_int, C.c_int, P(vp)]),
        "qvp_nccl_comm_destroy": (C.c_int, [vp]),
        "qvp_peer_group_create": (C.c_int, [C.c_int, C.c_int, sz, vp, P(vp)]),
        "qvp_peer_group_open": (C.c_int, [vp, vp]),
        "qvp_peer_group_destroy": (C.c_int, [vp]),
        "qvp_peer_group_output": (vp, [vp, C.c_uint64]),
        "qvp_shard_decode_peer": (C.c_int, [P(ShardDecodeArgs), vp, C.c_uint64, vp, vp]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


lib = _load()

# Every entry point include/qvp.h declares; tests check the library exports
# all of them.
EXPORTED = [
    "qvp_block_bytes", "qvp_block_stride", "qvp_last_error", "qvp_version", "qvp_device_sm_count",
    "qvp_pool_create", "qvp_pool_destroy", "qvp_pool_base", "qvp_pool_stride", "qvp_pool_num_blocks",
    "qvp_pool_device", "qvp_pool_write", "qvp_pool_read", "qvp_decode_workspace_size",
    "qvp_decode_plan", "qvp_decode", "qvp_decode_noalloc", "qvp_prefill", "qvp_copy_blocks", "qvp_gather_blocks", "qvp_scatter_blocks",
    "qvp_swap_slot_bytes", "qvp_compress_blocks", "qvp_decompress_blocks", "qvp_fetch_host",
    "qvp_kv_append", "qvp_shard_gather_bytes", "qvp_shard_decode", "qvp_shard_reassemble",
    "qvp_nccl_unique_id", "qvp_nccl_comm_init", "qvp_nccl_comm_destroy",
    "qvp_peer_group_create", "qvp_peer_group_open", "qvp_peer_group_destroy", "qvp_peer_group_output",
    "qvp_shard_decode_peer",
]


def last_error() -> str:
    return (lib.qvp_last_error() or b"").decode()


def check(status: int, what: str) -> None:
    if status != OK:
        raise QvpError(status, what)


def block_bytes(shape: BlockShape) -> int:
    return lib.qvp_block_bytes(C.byref(shape))


def block_stride(shape: BlockShape) -> int:
    return lib.qvp_block_stride(C.byref(shape))


def make_shape(tokens_per_block, num_layers, num_kv_heads, head_dim, bytes_per_element) -> BlockShape:
    return BlockShape(tokens_per_block, num_layers, num_kv_heads, head_dim, bytes_per_element)


class Pool:
    """One cudaMalloc'd block pool on `device` (zero-filled at creation)."""

    def __init__(self, shape: BlockShape, num_blocks: int, device: int = -1):
        self.shape = shape
        h = C.c_void_p()
        check(lib.qvp_pool_create(device, C.byref(shape), num_blocks, C.byref(h)), "qvp_pool_create")
        self.handle = h
        self.base = lib.qvp_pool_base(h)
        self.stride = lib.qvp_pool_stride(h)
        self.num_blocks = num_blocks

    def write(self, block: int, offset: int, data: bytes | memoryview) -> None:
        buf = (C.c_char * len(data)).from_buffer_copy(data)
        check(lib.qvp_pool_write(self.handle, block, offset, buf, len(data)), "qvp_pool_write")

    def read(self, block: int, offset: int, n: int) -> bytes:
        buf = (C.c_char * n)()
        check(lib.qvp_pool_read(self.handle, block, offset, buf, n), "qvp_pool_read")
        return bytes(buf)

    def close(self) -> None:
        if self.handle:
            check(lib.qvp_pool_destroy(self.handle), "qvp_pool_destroy")
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def decode_args(*, pool, block_stride, num_blocks, shape, dtype, layer, num_query_heads, scale, batch,
                max_blocks_per_seq, max_context_len, block_tables, context_lens, query, out,
                split_tokens=0, workspace=0, workspace_bytes=0, error_word=0) -> DecodeArgs:
    return DecodeArgs(pool, block_stride, num_blocks, shape, dtype, layer, num_query_heads, scale, batch,
                      max_blocks_per_seq, max_context_len, block_tables, context_lens, query, out,
                      split_tokens, workspace or None, workspace_bytes, error_word or None)


def decode_plan(args: DecodeArgs):
    split, ns, fast = C.c_uint32(), C.c_uint32(), C.c_int()
    check(lib.qvp_decode_plan(C.byref(args), C.byref(split), C.byref(ns), C.byref(fast)), "qvp_decode_plan")
    ws = C.c_size_t()
    check(lib.qvp_decode_workspace_size(C.byref(args), C.byref(ws)), "qvp_decode_workspace_size")
    return {"split_tokens": split.value, "num_splits": ns.value, "fast": bool(fast.value),
            "stream": fast.value == 2,
            "workspace_bytes": ws.value}


def decode(args: DecodeArgs, stream: int = 0) -> int:
    """Enqueues one batched decode; returns the status (does not raise)."""
    return lib.qvp_decode(C.byref(args), stream or None)


def nccl_unique_id() -> bytes:
    """A fresh NCCL unique id (make it on one rank, hand it to the others)."""
    buf = (C.c_char * NCCL_ID_BYTES)()
    check(lib.qvp_nccl_unique_id(buf, NCCL_ID_BYTES), "qvp_nccl_unique_id")
    return bytes(buf)


def nccl_comm_init(uid: bytes, nranks: int, rank: int) -> int:
    """An NCCL communicator on the current device (blocks until all join)."""
    buf = (C.c_char * len(uid)).from_buffer_copy(uid)
    comm = C.c_void_p()
    check(lib.qvp_nccl_comm_init(buf, len(uid), nranks, rank, C.byref(comm)), "qvp_nccl_comm_init")
    return comm.value


def nccl_comm_destroy(comm: int) -> None:
    check(lib.qvp_nccl_comm_destroy(comm), "qvp_nccl_comm_destroy")


def shard_decode_args(decode: DecodeArgs, shard: int, num_shards: int, device: int, comm, gathered, out):
    return ShardDecodeArgs(Shard(shard, num_shards, device), decode, comm or None, gathered, out)


def shard_gather_bytes(args: ShardDecodeArgs) -> int:
    n = C.c_size_t()
    check(lib.qvp_shard_gather_bytes(C.byref(args), C.byref(n)), "qvp_shard_gather_bytes")
    return n.value


class PeerGroup:
    """Output exchange over NVLink peer memory for kv-head shards: create on
    every rank, exchange `handle` (bytes) by any transport, then open with
    every rank's handle in rank order."""

    def __init__(self, rank: int, nranks: int, out_bytes: int):
        buf = (C.c_char * PEER_HANDLE_BYTES)()
        g = C.c_void_p()
        check(lib.qvp_peer_group_create(rank, nranks, out_bytes, buf, C.byref(g)), "qvp_peer_group_create")
        self.handle_ptr = g
        self.handle = bytes(buf)

    def open(self, handles: list) -> None:
        blob = b"".join(handles)
        buf = (C.c_char * len(blob)).from_buffer_copy(blob)
        check(lib.qvp_peer_group_open(self.handle_ptr, buf), "qvp_peer_group_open")

    def output(self, step: int) -> int:
        return lib.qvp_peer_group_output(self.handle_ptr, step)

    def decode(self, args: ShardDecodeArgs, step: int, error_word: int, stream: int) -> int:
        return lib.qvp_shard_decode_peer(C.byref(args), self.handle_ptr, step, error_word or None, stream or None)

    def close(self) -> None:
        if self.handle_ptr:
            check(lib.qvp_peer_group_destroy(self.handle_ptr), "qvp_peer_group_destroy")
            self.handle_ptr = None
