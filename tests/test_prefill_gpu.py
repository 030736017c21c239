"""GPU parity checks of qvp_prefill against the prefill oracle (the
reference's decode at every prompt position)."""
import numpy as np
import pytest

import oracle
import workloads as W

pytestmark = pytest.mark.gpu

BF16_ABS = 2e-2
F32_REL = 1e-5


def gpu_prefill(w, pool, q, ql):
    import ctypes as C

    import torch

    import qvp
    dev = torch.device("cuda", 0)
    bf = w.dtype == "bf16"
    pool_d = torch.from_numpy(np.ascontiguousarray(pool)).to(dev)
    q_d = torch.from_numpy(np.ascontiguousarray(q).view(np.int16 if bf else np.float32)).to(dev)
    out_d = torch.zeros_like(q_d)
    tab = torch.from_numpy(np.ascontiguousarray(w.tables)).to(dev)
    ctx = torch.from_numpy(np.ascontiguousarray(w.context_lens)).to(dev)
    qld = torch.from_numpy(np.ascontiguousarray(ql, dtype=np.int32)).to(dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    a = qvp.PrefillArgs()
    a.pool, a.block_stride, a.num_blocks = pool_d.data_ptr(), w.block_stride, w.num_blocks
    a.shape = qvp.make_shape(w.tokens_per_block, w.num_layers, w.num_kv_heads, w.head_dim, w.elem)
    a.dtype = qvp.DTYPE_BF16 if bf else qvp.DTYPE_F32
    a.layer, a.num_query_heads, a.scale, a.batch = w.layer, w.num_query_heads, w.scale, w.batch
    a.max_blocks_per_seq, a.max_query_len = w.pitch, q.shape[1]
    a.block_tables, a.context_lens, a.query_lens = tab.data_ptr(), ctx.data_ptr(), qld.data_ptr()
    a.query, a.out, a.error_word = q_d.data_ptr(), out_d.data_ptr(), err.data_ptr()
    st = qvp.lib.qvp_prefill(C.byref(a), torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    o = out_d.view(torch.bfloat16).float() if bf else out_d.view(torch.float32)
    return st, o.cpu().numpy(), int(err.item())


@pytest.mark.parametrize("kw", [
    dict(hq=28, hkv=4, head_dim=128, dtype="bf16"),   # fast path, G = 7 (18-token tiles)
    dict(hq=64, hkv=8, head_dim=128, dtype="bf16"),   # G = 8
    dict(hq=16, hkv=1, head_dim=64, dtype="bf16"),    # G = 16, head_dim 64
    dict(hq=4, hkv=4, head_dim=128, dtype="bf16"),    # G = 1 (128-token tiles)
    dict(hq=8, hkv=2, head_dim=64, dtype="f32"),      # generic path
])
def test_prefill_matches_per_position_decode(kw):
    w = W.small(71, batch=4, ctx_lo=1, ctx_hi=400, **kw)
    rng = np.random.default_rng(5)
    ql = np.array([min(int(c), n) for c, n in zip(w.context_lens, (1, 37, 200, 400))], dtype=np.int32)
    pool, _ = W.host_inputs(w)
    qf = rng.standard_normal((w.batch, int(ql.max()), w.num_query_heads, w.head_dim), dtype=np.float32)
    q = W.f32_to_bf16_bits(qf) if w.dtype == "bf16" else qf
    ref, status = oracle.port_prefill(w, pool, q, ql, threads=8)
    assert status.all()
    st, out, err = gpu_prefill(w, pool, q, ql)
    assert st == 0 and err == 0
    for b in range(w.batch):
        got, want = out[b, : ql[b]], ref[b, : ql[b]]
        if w.dtype == "bf16":
            assert np.max(np.abs(got - want)) < BF16_ABS
        else:
            assert np.max(np.abs(got - want)) <= F32_REL * max(1.0, float(np.abs(want).max()))
