"""CPU checks of libqvp.so: it loads, exports every entry point include/qvp.h
declares, and rejects inconsistent decode arguments on the host (no device
work is reached, so these run without a GPU)."""
import ctypes as C
import os
import re

import pytest

import qvp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    text = open(os.path.join(ROOT, "include", "qvp.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(qvp_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_entry_point():
    names = declared_symbols()
    assert len(names) >= 20
    for n in names:
        assert hasattr(qvp.lib, n), n
    assert set(names) == set(qvp.EXPORTED)


def test_version_string():
    assert b"sm_100a" in qvp.lib.qvp_version()


def test_block_bytes_and_stride_match_the_reference_rounding():
    # BlockShape::byte_size (src/Block.cpp:8-13) and the 256-byte rounding of
    # every block allocation (src/Block.cpp:30-44).
    s = qvp.make_shape(16, 1, 4, 128, 2)
    assert qvp.block_bytes(s) == 16 * 4 * 128 * 2 * 2 == 32768
    assert qvp.block_stride(s) == 32768
    s = qvp.make_shape(4, 1, 1, 4, 4)
    assert qvp.block_bytes(s) == 128 and qvp.block_stride(s) == 256
    s = qvp.make_shape(0, 1, 1, 4, 4)
    assert qvp.block_bytes(s) == 0 and qvp.block_stride(s) == 256


def _args(**kw):
    base = dict(pool=0x1000, block_stride=256, num_blocks=4, shape=qvp.make_shape(4, 1, 1, 4, 4),
                dtype=qvp.DTYPE_F32, layer=0, num_query_heads=1, scale=1.0, batch=1, max_blocks_per_seq=1,
                max_context_len=4, block_tables=0x2000, context_lens=0x3000, query=0x4000, out=0x5000)
    base.update(kw)
    return qvp.decode_args(**base)


@pytest.mark.parametrize("bad", [
    dict(shape=qvp.make_shape(4, 1, 1, 4, 8)),          # element size mismatch (double vs float)
    dict(dtype=qvp.DTYPE_BF16),                          # bf16 over a 4-byte shape
    dict(layer=1),                                       # layer beyond the block shape
    dict(num_query_heads=0),                             # zero query heads
    dict(shape=qvp.make_shape(4, 1, 2, 4, 4), num_query_heads=3),  # heads that do not group
    dict(max_context_len=0),                             # zero context
    dict(max_context_len=5),                             # context longer than the mapped blocks
    dict(query=0),                                       # null query
    dict(out=0),                                         # null output
    dict(block_stride=64),                               # stride below the block size
])
def test_decode_rejects_inconsistent_arguments_before_any_launch(bad):
    a = _args(**bad)
    assert qvp.decode(a) == qvp.ERR_INVALID
    assert qvp.last_error()


def test_decode_plan_splits_long_contexts():
    a = _args(shape=qvp.make_shape(16, 1, 4, 128, 2), dtype=qvp.DTYPE_BF16, block_stride=32768,
              num_query_heads=28, batch=64, max_blocks_per_seq=512, max_context_len=8192, split_tokens=512)
    p = qvp.decode_plan(a)
    assert p["fast"] and p["split_tokens"] == 512 and p["num_splits"] == 16
    assert p["workspace_bytes"] >= 64 * 16 * 28 * (128 + 2) * 4
    a.split_tokens = 100  # not a multiple of the 16-token block
    assert qvp.decode(a) == qvp.ERR_INVALID


def test_decode_plan_falls_back_to_the_generic_kernel_for_other_shapes():
    p = qvp.decode_plan(_args())
    assert not p["fast"] and p["num_splits"] == 1 and p["workspace_bytes"] == 0
    # padded blocks (stride > byte size) cannot use the TMA view of the pool
    a = _args(shape=qvp.make_shape(16, 1, 1, 64, 2), dtype=qvp.DTYPE_BF16, block_stride=4096 + 256,
              max_blocks_per_seq=1, max_context_len=16)
    assert not qvp.decode_plan(a)["fast"]


def test_workspace_too_small_is_refused():
    a = _args(shape=qvp.make_shape(16, 1, 4, 128, 2), dtype=qvp.DTYPE_BF16, block_stride=32768,
              num_query_heads=28, batch=2, max_blocks_per_seq=64, max_context_len=1024, split_tokens=256)
    assert qvp.decode(a) == qvp.ERR_WORKSPACE


@pytest.mark.parametrize("split", [0, 256])  # stream-K records and split-K partials
def test_misaligned_workspace_is_refused_before_any_launch(split):
    a = _args(shape=qvp.make_shape(16, 1, 4, 128, 2), dtype=qvp.DTYPE_BF16, block_stride=32768,
              num_query_heads=28, batch=2, max_blocks_per_seq=64, max_context_len=1024, split_tokens=split)
    need = qvp.decode_plan(a)["workspace_bytes"]
    assert need > 0
    a.workspace, a.workspace_bytes = 0x10008, need + 64
    assert qvp.decode(a) == qvp.ERR_WORKSPACE
    assert "aligned" in qvp.last_error()


def test_movers_reject_bad_arguments():
    lib = qvp.lib
    assert lib.qvp_copy_blocks(None, 256, 4, 256, None, 1, None, None) == qvp.ERR_INVALID
    assert lib.qvp_copy_blocks(C.c_void_p(0x1000), 256, 4, 512, C.c_void_p(0x2000), 1, None, None) == qvp.ERR_INVALID
    assert lib.qvp_copy_blocks(None, 256, 4, 256, None, 0, None, None) == qvp.OK  # empty batch
    assert lib.qvp_gather_blocks(None, 256, 4, 256, None, 1, None, None, None) == qvp.ERR_INVALID
    assert lib.qvp_scatter_blocks(None, 256, 4, 256, None, 1, None, None, None) == qvp.ERR_INVALID
    s = qvp.make_shape(4, 1, 1, 4, 4)
    assert lib.qvp_kv_append(None, 256, 4, C.byref(s), 0, 1, 1, None, None, None, None, None, None) == qvp.ERR_INVALID
    assert lib.qvp_kv_append(C.c_void_p(1), 256, 4, C.byref(s), 1, 1, 1, C.c_void_p(1), C.c_void_p(1),
                             C.c_void_p(1), C.c_void_p(1), None, None) == qvp.ERR_INVALID


def test_shard_gather_bytes_and_refusals_on_the_host():
    a = _args(shape=qvp.make_shape(16, 1, 1, 128, 2), dtype=qvp.DTYPE_BF16, block_stride=8192,
              num_query_heads=7, batch=64, max_blocks_per_seq=4, max_context_len=64)
    sa = qvp.shard_decode_args(a, 1, 4, -1, None, 0, 0)
    # four slots of [64][7][128] bf16
    assert qvp.shard_gather_bytes(sa) == 4 * 64 * 7 * 128 * 2
    n = C.c_size_t()
    bad = qvp.shard_decode_args(a, 4, 4, -1, None, 0, 0)
    assert qvp.lib.qvp_shard_gather_bytes(C.byref(bad), C.byref(n)) == qvp.ERR_INVALID
    assert qvp.lib.qvp_shard_reassemble(None, None, 0, 1, 1, 1, 2, None) == qvp.ERR_INVALID
    # nothing to move: no launch, no error
    assert qvp.lib.qvp_shard_reassemble(None, None, 2, 0, 7, 128, 2, None) == qvp.OK
    assert qvp.lib.qvp_nccl_comm_init(None, 0, 2, 0, C.byref(C.c_void_p())) == qvp.ERR_INVALID
    assert qvp.lib.qvp_nccl_comm_destroy(None) == qvp.OK
