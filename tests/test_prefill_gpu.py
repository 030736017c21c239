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


def _prefill_case(seed, qscale=1.0, poison_tail=False, **kw):
    w = W.small(seed, **kw)
    rng = np.random.default_rng(seed)
    ql = np.minimum(w.context_lens, rng.integers(1, 700, size=w.batch)).astype(np.int32)
    ql[0] = w.context_lens[0]  # one whole-prompt prefill
    pool, _ = W.host_inputs(w)
    if poison_tail:
        # NaN in every K and V slot past each context: the kernel must not read them into its sums
        v = pool.view(np.uint16).reshape(w.num_blocks, -1)
        per_tok = w.num_kv_heads * w.head_dim
        for b in range(w.batch):
            c = int(w.context_lens[b])
            if c % w.tokens_per_block == 0:
                continue
            blk = int(w.tables[b, c // w.tokens_per_block])
            for kv in range(2):
                base = (w.layer * 2 + kv) * w.tokens_per_block * per_tok
                v[blk, base + (c % w.tokens_per_block) * per_tok: base + w.tokens_per_block * per_tok] = 0x7FC0
    qf = rng.standard_normal((w.batch, int(ql.max()), w.num_query_heads, w.head_dim), dtype=np.float32) * qscale
    q = W.f32_to_bf16_bits(qf)
    ref, status = oracle.port_prefill(w, pool, q, ql, threads=8)
    assert status.all()
    st, out, err = gpu_prefill(w, pool, q, ql)
    assert st == 0 and err == 0
    for b in range(w.batch):
        got, want = out[b, : ql[b]], ref[b, : ql[b]]
        assert np.isfinite(got).all()
        assert np.max(np.abs(got - want)) < BF16_ABS, (b, float(np.max(np.abs(got - want))))


@pytest.mark.parametrize("hq,hkv", [(28, 4), (32, 8), (16, 16)])
def test_prefill_long_prompts_past_many_key_steps(hq, hkv):
    # contexts up to 1500 tokens: a tile runs up to 12 steps of 128 keys
    _prefill_case(81, batch=3, ctx_lo=900, ctx_hi=1500, hq=hq, hkv=hkv, head_dim=128, dtype="bf16")


def test_prefill_rescales_when_scores_grow():
    # large queries: row maxima jump by far more than 2^8 between key steps
    _prefill_case(82, qscale=24.0, batch=3, ctx_lo=300, ctx_hi=900, hq=28, hkv=4, head_dim=128, dtype="bf16")


def test_prefill_ignores_bytes_past_the_context():
    _prefill_case(83, poison_tail=True, batch=4, ctx_lo=17, ctx_hi=600, hq=28, hkv=4, head_dim=128, dtype="bf16")


def test_prefill_unaligned_rows_take_the_warp_kernel():
    """q and out 4-byte but not 16-byte aligned: the mma.sync kernel runs."""
    import ctypes as C

    import torch

    import qvp
    w = W.small(84, batch=2, ctx_lo=40, ctx_hi=300, hq=28, hkv=4, head_dim=128, dtype="bf16")
    ql = w.context_lens.astype(np.int32)
    pool, _ = W.host_inputs(w)
    rng = np.random.default_rng(84)
    q = W.f32_to_bf16_bits(rng.standard_normal((w.batch, int(ql.max()), w.num_query_heads, w.head_dim),
                                               dtype=np.float32))
    ref, status = oracle.port_prefill(w, pool, q, ql, threads=8)
    dev = torch.device("cuda", 0)
    n = q.size
    qbuf = torch.zeros(n + 8, dtype=torch.int16, device=dev)
    qbuf[2:2 + n] = torch.from_numpy(np.ascontiguousarray(q).view(np.int16).reshape(-1)).to(dev)
    obuf = torch.zeros(n + 8, dtype=torch.int16, device=dev)
    pool_d = torch.from_numpy(np.ascontiguousarray(pool)).to(dev)
    tab = torch.from_numpy(np.ascontiguousarray(w.tables)).to(dev)
    ctx = torch.from_numpy(np.ascontiguousarray(w.context_lens)).to(dev)
    qld = torch.from_numpy(ql).to(dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    a = qvp.PrefillArgs()
    a.pool, a.block_stride, a.num_blocks = pool_d.data_ptr(), w.block_stride, w.num_blocks
    a.shape = qvp.make_shape(w.tokens_per_block, w.num_layers, w.num_kv_heads, w.head_dim, w.elem)
    a.dtype = qvp.DTYPE_BF16
    a.layer, a.num_query_heads, a.scale, a.batch = w.layer, w.num_query_heads, w.scale, w.batch
    a.max_blocks_per_seq, a.max_query_len = w.pitch, q.shape[1]
    a.block_tables, a.context_lens, a.query_lens = tab.data_ptr(), ctx.data_ptr(), qld.data_ptr()
    a.query, a.out, a.error_word = qbuf.data_ptr() + 4, obuf.data_ptr() + 4, err.data_ptr()
    assert qvp.lib.qvp_prefill(C.byref(a), torch.cuda.current_stream().cuda_stream) == 0
    torch.cuda.synchronize()
    assert err.item() == 0
    out = obuf[2:2 + n].view(torch.bfloat16).float().cpu().numpy().reshape(q.shape)
    for b in range(w.batch):
        assert np.max(np.abs(out[b, : ql[b]] - ref[b, : ql[b]])) < BF16_ABS


def test_prefill_second_layer_of_two():
    _prefill_case(85, batch=3, ctx_lo=100, ctx_hi=500, hq=28, hkv=4, head_dim=128, dtype="bf16", num_layers=2,
                  layer=1)
