"""GPU test of qvp_decode_noalloc, the decode entry point for callers that
cannot allocate device memory (a host that owns the whole HBM budget, an FFI
caller with no device allocator, a step loop where cudaMalloc would
synchronise the device). Its scratch is a fixed 16 MiB array inside the
library; it must give outputs identical (bit for bit) to qvp_decode with a caller
workspace, call after call, whatever the array held before, and refuse batches whose scratch would not fit.

Named test_zz_* so pytest collects it last.
"""
import ctypes as C

import numpy as np
import pytest

import qvp
import workloads as W
from helpers import gpu_decode

pytestmark = pytest.mark.gpu

STATIC_SCRATCH = 16 << 20


def _device_args(w, pool, q, split_tokens=0):
    import torch
    dev = torch.device("cuda", 0)
    bufs = {
        "pool": torch.from_numpy(np.ascontiguousarray(pool)).to(dev),
        "q": torch.from_numpy(np.ascontiguousarray(q).view(np.int16 if w.dtype == "bf16" else np.float32)).to(dev),
        "ctx": torch.from_numpy(np.ascontiguousarray(w.context_lens)).to(dev),
        "tab": torch.from_numpy(np.ascontiguousarray(w.tables)).to(dev),
        "err": torch.zeros(1, dtype=torch.int32, device=dev),
    }
    out_dtype = torch.bfloat16 if w.dtype == "bf16" else torch.float32
    bufs["out"] = torch.zeros((w.batch, w.num_query_heads, w.head_dim), dtype=out_dtype, device=dev)
    shape = qvp.make_shape(w.tokens_per_block, w.num_layers, w.num_kv_heads, w.head_dim, w.elem)
    a = qvp.decode_args(pool=bufs["pool"].data_ptr(), block_stride=w.block_stride, num_blocks=w.num_blocks,
                        shape=shape, dtype=qvp.DTYPE_F32 if w.dtype == "f32" else qvp.DTYPE_BF16, layer=w.layer,
                        num_query_heads=w.num_query_heads, scale=w.scale, batch=w.batch,
                        max_blocks_per_seq=w.pitch, max_context_len=w.max_context_len,
                        block_tables=bufs["tab"].data_ptr(), context_lens=bufs["ctx"].data_ptr(),
                        query=bufs["q"].data_ptr(), out=bufs["out"].data_ptr(), split_tokens=split_tokens,
                        error_word=bufs["err"].data_ptr())
    return a, bufs


def _case(name):
    if name == "bf16-stream-k":
        return W.small(31, batch=16, ctx_lo=1, ctx_hi=3000, hq=28, hkv=4, head_dim=128, dtype="bf16"), 0
    if name == "bf16-stream-k-large":
        return W.small(34, batch=96, ctx_lo=500, ctx_hi=6000, hq=28, hkv=4, head_dim=128, dtype="bf16"), 0
    if name == "bf16-grid-split":
        return W.small(32, batch=8, ctx_lo=100, ctx_hi=2500, hq=28, hkv=4, head_dim=128, dtype="bf16"), 256
    return W.cfg1(), 48


def _check_calls(name, calls=2):
    """Runs `name` through qvp_decode (caller workspace) once and through
    qvp_decode_noalloc `calls` times; the kernels and the plan are the same,
    so the outputs must be identical bit for bit."""
    import torch
    w, split = _case(name)
    pool, q = W.host_inputs(w)
    st, want, err, plan = gpu_decode(w, pool, q, split_tokens=split)   # caller-workspace entry point
    assert st == 0 and err == 0
    assert 0 < plan["workspace_bytes"] <= STATIC_SCRATCH

    a, bufs = _device_args(w, pool, q, split)
    stream = torch.cuda.current_stream().cuda_stream
    for call in range(calls):
        bufs["out"].fill_(-7.0)
        assert qvp.lib.qvp_decode_noalloc(C.byref(a), stream) == 0, qvp.last_error()
        torch.cuda.synchronize()
        got = bufs["out"].float().cpu().numpy()
        assert int(bufs["err"].item()) == 0
        assert np.array_equal(got, want), (name, call, float(np.max(np.abs(got - want))))
    return plan["workspace_bytes"]


@pytest.mark.parametrize("case", ["bf16-stream-k", "bf16-grid-split", "fp32-generic-split"])
def test_no_alloc_decode_matches_qvp_decode_on_two_calls_in_a_row(case):
    _check_calls(case)


def test_no_alloc_decode_after_a_larger_call_ignores_stale_scratch():
    # the larger batch leaves records all over the shared array; the smaller
    # one that follows must not read any of them
    big = _check_calls("bf16-stream-k-large", calls=1)
    small = _check_calls("bf16-stream-k", calls=2)
    assert big > small


def test_no_alloc_decode_refuses_batches_beyond_its_scratch():
    import torch
    w = W.small(33, batch=700, ctx_lo=4000, ctx_hi=4096, hq=28, hkv=4, head_dim=128, dtype="bf16",
                pool_factor=1.0)
    # a forced 256-token split of 700 long contexts needs far more than 16 MiB
    shape = qvp.make_shape(16, 1, 4, 128, 2)
    dummy = torch.zeros(16, dtype=torch.uint8, device="cuda")
    a = qvp.decode_args(pool=dummy.data_ptr(), block_stride=32768, num_blocks=w.num_blocks, shape=shape,
                        dtype=qvp.DTYPE_BF16, layer=0, num_query_heads=28, scale=w.scale, batch=w.batch,
                        max_blocks_per_seq=w.pitch, max_context_len=w.max_context_len,
                        block_tables=dummy.data_ptr(), context_lens=dummy.data_ptr(), query=dummy.data_ptr(),
                        out=dummy.data_ptr(), split_tokens=256)
    need = qvp.decode_plan(a)["workspace_bytes"]
    assert need > STATIC_SCRATCH  # guard: the call below must be refused on the host
    assert qvp.lib.qvp_decode_noalloc(C.byref(a), None) == qvp.ERR_WORKSPACE
    assert "static array" in qvp.last_error()
