"""KV-head sharding through the C ABI on the GPU (qvp_shard_decode,
qvp_shard_reassemble, the NCCL helpers).

Every GQA group is independent (PagedAttention.h:94-96), so shard r of n
decodes kv heads [r*Hkv/n, (r+1)*Hkv/n) from a pool that holds only those
heads, with the same block ids and tables as every other shard.

One GPU: the n shard decodes of one batch run one after another into the
slots of one gather buffer and qvp_shard_reassemble puts the heads back in
order. The result must equal the shard outputs concatenated along the heads
bit for bit (the reorder moves bytes only), match the oracle within the bf16
tolerance, and match the unsharded qvp_decode within the same tolerance. It
cannot match it bit for bit: a CTA of the unsharded decode streams 4 kv heads
and spreads each head's blocks over 2 warps, a 1-head shard spreads them over
8, so the fp32 partial sums are added in a different order.

Two or more GPUs: one process per GPU, a communicator made by libqvp, and
qvp_shard_decode's in-place NCCL all-gather; every rank must end with the
whole [B, Hq, D] output. Skipped when fewer than two GPUs are visible.
"""
import ctypes as C
import os

import numpy as np
import pytest

import oracle
import qvp
import sharding
import workloads as W
from helpers import device_bytes, gpu_decode

pytestmark = pytest.mark.gpu

BF16_ABS = 2e-2


def _decode_args(sw, pool_d, q_d, out_ptr, tab_d, ctx_d, err_d):
    shape = qvp.make_shape(sw.tokens_per_block, sw.num_layers, sw.num_kv_heads, sw.head_dim, sw.elem)
    return qvp.decode_args(pool=pool_d.data_ptr(), block_stride=sw.block_stride, num_blocks=sw.num_blocks,
                           shape=shape, dtype=qvp.DTYPE_BF16 if sw.dtype == "bf16" else qvp.DTYPE_F32,
                           layer=sw.layer, num_query_heads=sw.num_query_heads, scale=sw.scale, batch=sw.batch,
                           max_blocks_per_seq=sw.pitch, max_context_len=sw.max_context_len,
                           block_tables=tab_d.data_ptr(), context_lens=ctx_d.data_ptr(), query=q_d.data_ptr(),
                           out=out_ptr, error_word=err_d.data_ptr())


def _with_workspace(a, dev, keep):
    import torch
    plan = qvp.decode_plan(a)
    if plan["workspace_bytes"]:
        ws = torch.empty(plan["workspace_bytes"], dtype=torch.uint8, device=dev)
        keep.append(ws)
        a.workspace, a.workspace_bytes = ws.data_ptr(), plan["workspace_bytes"]
    return plan


def _shard_inputs(w, pool, q, n, r, dev):
    import torch
    sw = sharding.shard_workload(w, n)
    sp = sharding.shard_pool(pool, w, n, r)
    sq = sharding.shard_query(q, w.num_kv_heads, n, r)
    pool_d = torch.from_numpy(sp).to(dev)
    q_d = torch.from_numpy(sq.view(np.int16) if w.dtype == "bf16" else sq).to(dev)
    return sw, pool_d, q_d


@pytest.mark.parametrize("n", [2, 4])
def test_shards_on_one_gpu_reassemble_to_the_unsharded_decode(n):
    import torch
    dev = torch.device("cuda", 0)
    w = W.small(51, batch=12, ctx_lo=1, ctx_hi=3000, hq=28, hkv=4, head_dim=128, dtype="bf16")
    pool, q = W.host_inputs(w)
    hs = w.num_query_heads // n
    slot = w.batch * hs * w.head_dim * 2
    gathered = torch.empty(n * slot, dtype=torch.uint8, device=dev)
    full = torch.empty((w.batch, w.num_query_heads, w.head_dim), dtype=torch.bfloat16, device=dev)
    tab_d = torch.from_numpy(w.tables).to(dev)
    ctx_d = torch.from_numpy(w.context_lens).to(dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    keep = []
    st = torch.cuda.current_stream().cuda_stream
    for r in range(n):
        sw, pool_d, q_d = _shard_inputs(w, pool, q, n, r, dev)
        keep += [pool_d, q_d]
        a = _decode_args(sw, pool_d, q_d, gathered.data_ptr() + r * slot, tab_d, ctx_d, err)
        plan = _with_workspace(a, dev, keep)
        assert plan["stream"]
        assert qvp.decode(a, st) == 0, qvp.last_error()
        torch.cuda.synchronize()  # the shards share nothing but may reuse one workspace
    assert qvp.lib.qvp_shard_reassemble(gathered.data_ptr(), full.data_ptr(), n, w.batch, hs, w.head_dim, 2,
                                        st) == 0, qvp.last_error()
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    got = full.float().cpu().numpy()
    parts = gathered.view(torch.bfloat16).view(n, w.batch, hs, w.head_dim).float().cpu().numpy()
    assert np.array_equal(got, np.concatenate(list(parts), axis=1))
    ref, status = oracle.port_decode(w, pool, q, threads=8)
    assert status.all()
    assert np.max(np.abs(got - ref)) < BF16_ABS
    st_u, unsharded, err_u, _ = gpu_decode(w, pool, q)
    assert st_u == 0 and err_u == 0
    assert np.max(np.abs(got - unsharded)) < BF16_ABS


def test_one_shard_decode_is_qvp_decode_bit_for_bit():
    import torch
    dev = torch.device("cuda", 0)
    w = W.small(52, batch=9, ctx_lo=1, ctx_hi=2500, hq=28, hkv=4, head_dim=128, dtype="bf16")
    pool, q = W.host_inputs(w)
    st_u, want, err_u, _ = gpu_decode(w, pool, q)
    assert st_u == 0 and err_u == 0
    sw, pool_d, q_d = _shard_inputs(w, pool, q, 1, 0, dev)
    tab_d = torch.from_numpy(w.tables).to(dev)
    ctx_d = torch.from_numpy(w.context_lens).to(dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    out = torch.full((w.batch, w.num_query_heads, w.head_dim), -3.0, dtype=torch.bfloat16, device=dev)
    keep = []
    # decode.out only has to be non-null: the shard decode writes the gather buffer
    a = _decode_args(sw, pool_d, q_d, out.data_ptr(), tab_d, ctx_d, err)
    _with_workspace(a, dev, keep)
    sa = qvp.shard_decode_args(a, 0, 1, 0, None, 0, out.data_ptr())
    gathered = torch.empty(qvp.shard_gather_bytes(sa), dtype=torch.uint8, device=dev)
    sa.gathered = gathered.data_ptr()
    assert qvp.lib.qvp_shard_decode(C.byref(sa), torch.cuda.current_stream().cuda_stream) == 0, qvp.last_error()
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert np.array_equal(out.float().cpu().numpy(), want)


def test_shard_decode_refuses_a_shard_on_another_device_or_without_a_communicator():
    import torch
    dev = torch.device("cuda", 0)
    w = W.small(53, batch=2, ctx_lo=1, ctx_hi=100, hq=28, hkv=4, head_dim=128, dtype="bf16")
    pool, q = W.host_inputs(w)
    sw, pool_d, q_d = _shard_inputs(w, pool, q, 2, 0, dev)
    tab_d = torch.from_numpy(w.tables).to(dev)
    ctx_d = torch.from_numpy(w.context_lens).to(dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    out = torch.zeros((w.batch, w.num_query_heads, w.head_dim), dtype=torch.bfloat16, device=dev)
    a = _decode_args(sw, pool_d, q_d, 0, tab_d, ctx_d, err)
    sa = qvp.shard_decode_args(a, 0, 2, 0, None, out.data_ptr(), out.data_ptr())
    assert qvp.lib.qvp_shard_decode(C.byref(sa), None) == qvp.ERR_INVALID
    assert "communicator" in qvp.last_error()
    sa = qvp.shard_decode_args(a, 0, 1, torch.cuda.device_count() + 3, None, out.data_ptr(), out.data_ptr())
    assert qvp.lib.qvp_shard_decode(C.byref(sa), None) == qvp.ERR_INVALID
    assert "device" in qvp.last_error()


# --- real NCCL over two or more GPUs --------------------------------------------

def _rank_main(rank, world, uid_path, result):
    import time

    import torch
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    if rank == 0:
        uid = qvp.nccl_unique_id()
        with open(uid_path + ".tmp", "wb") as f:
            f.write(uid)
        os.rename(uid_path + ".tmp", uid_path)
    else:
        t0 = time.time()
        while not os.path.exists(uid_path):
            if time.time() - t0 > 60:
                result[rank] = "no unique id"
                return
            time.sleep(0.05)
        with open(uid_path, "rb") as f:
            uid = f.read()
    comm = qvp.nccl_comm_init(uid, world, rank)
    w = W.small(54, batch=10, ctx_lo=1, ctx_hi=4000, hq=28, hkv=4, head_dim=128, dtype="bf16")
    pool, q = W.host_inputs(w)
    sw, pool_d, q_d = _shard_inputs(w, pool, q, world, rank, dev)
    tab_d = torch.from_numpy(w.tables).to(dev)
    ctx_d = torch.from_numpy(w.context_lens).to(dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    out = torch.zeros((w.batch, w.num_query_heads, w.head_dim), dtype=torch.bfloat16, device=dev)
    keep = []
    a = _decode_args(sw, pool_d, q_d, out.data_ptr(), tab_d, ctx_d, err)
    _with_workspace(a, dev, keep)
    sa = qvp.shard_decode_args(a, rank, world, rank, comm, 0, out.data_ptr())
    gathered = torch.empty(qvp.shard_gather_bytes(sa), dtype=torch.uint8, device=dev)
    sa.gathered = gathered.data_ptr()
    st = torch.cuda.current_stream().cuda_stream
    outs = []
    for _ in range(2):  # two steps in a row through the same buffers
        out.zero_()
        rc = qvp.lib.qvp_shard_decode(C.byref(sa), st)
        if rc != 0:
            result[rank] = f"qvp_shard_decode {rc}: {qvp.last_error()}"
            return
        torch.cuda.synchronize()
        outs.append(out.float().cpu().numpy())
    torch.cuda.synchronize()
    qvp.nccl_comm_destroy(comm)
    ref, status = oracle.port_decode(w, pool, q, threads=4)
    ok = (int(err.item()) == 0 and status.all() and np.array_equal(outs[0], outs[1])
          and float(np.max(np.abs(outs[0] - ref))) < BF16_ABS)
    result[rank] = "ok" if ok else f"mismatch: err {int(err.item())} max {float(np.max(np.abs(outs[0] - ref)))}"


def test_nccl_all_gather_gives_every_rank_every_head(tmp_path):
    import torch
    import torch.multiprocessing as mp
    world = min(torch.cuda.device_count(), 4)
    if world < 2:
        pytest.skip("needs two GPUs")
    mgr = mp.Manager()
    result = mgr.dict()
    ctx = mp.get_context("spawn")
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    procs = [ctx.Process(target=_rank_main, args=(r, world, str(tmp_path / "uid"), result)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:  # host processes only: nothing is left running on a GPU
        p.kill()
    assert not alive
    assert [result.get(r) for r in range(world)] == ["ok"] * world


# --- output exchange over NVLink peer memory -----------------------------------

def test_peer_group_of_one_gpu_is_qvp_decode_bit_for_bit():
    import torch
    dev = torch.device("cuda", 0)
    w = W.small(55, batch=9, ctx_lo=1, ctx_hi=2500, hq=28, hkv=4, head_dim=128, dtype="bf16")
    pool, q = W.host_inputs(w)
    st_u, want, err_u, _ = gpu_decode(w, pool, q)
    assert st_u == 0 and err_u == 0
    sw, pool_d, q_d = _shard_inputs(w, pool, q, 1, 0, dev)
    tab_d = torch.from_numpy(w.tables).to(dev)
    ctx_d = torch.from_numpy(w.context_lens).to(dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    keep = []
    a = _decode_args(sw, pool_d, q_d, q_d.data_ptr(), tab_d, ctx_d, err)
    _with_workspace(a, dev, keep)
    g = qvp.PeerGroup(0, 1, w.batch * w.num_query_heads * w.head_dim * 2)
    g.open([g.handle])
    sa = qvp.shard_decode_args(a, 0, 1, 0, None, 0, 0)
    st = torch.cuda.current_stream().cuda_stream
    for step in range(3):
        assert g.decode(sa, step, err.data_ptr(), st) == 0, qvp.last_error()
        torch.cuda.synchronize()
        got = torch.empty((w.batch, w.num_query_heads, w.head_dim), dtype=torch.bfloat16, device=dev)
        got.view(-1).view(torch.uint8).copy_(device_bytes(g.output(step), got.numel() * 2, dev))
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        assert np.array_equal(got.float().cpu().numpy(), want), step
    g.close()


def _peer_rank_main(rank, world, tmp, result):
    import time

    import torch
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    w = W.small(56, batch=10, ctx_lo=1, ctx_hi=4000, hq=28, hkv=4, head_dim=128, dtype="bf16")
    pool, q = W.host_inputs(w)
    nbytes = w.batch * w.num_query_heads * w.head_dim * 2
    g = qvp.PeerGroup(rank, world, nbytes)
    with open(os.path.join(tmp, f"h{rank}.tmp"), "wb") as f:
        f.write(g.handle)
    os.rename(os.path.join(tmp, f"h{rank}.tmp"), os.path.join(tmp, f"h{rank}"))
    t0 = time.time()
    while not all(os.path.exists(os.path.join(tmp, f"h{r}")) for r in range(world)):
        if time.time() - t0 > 60:
            result[rank] = "no handles"
            return
        time.sleep(0.05)
    g.open([open(os.path.join(tmp, f"h{r}"), "rb").read() for r in range(world)])
    sw, pool_d, q_d = _shard_inputs(w, pool, q, world, rank, dev)
    tab_d = torch.from_numpy(w.tables).to(dev)
    ctx_d = torch.from_numpy(w.context_lens).to(dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    keep = []
    a = _decode_args(sw, pool_d, q_d, q_d.data_ptr(), tab_d, ctx_d, err)
    _with_workspace(a, dev, keep)
    sa = qvp.shard_decode_args(a, rank, world, rank, None, 0, 0)
    st = torch.cuda.current_stream().cuda_stream
    ref, status = oracle.port_decode(w, pool, q, threads=4)
    msg = "ok"
    for step in range(4):  # both buffers, twice
        rc = g.decode(sa, step, err.data_ptr(), st)
        if rc != 0:
            msg = f"qvp_shard_decode_peer {rc}: {qvp.last_error()}"
            break
        got = torch.empty((w.batch, w.num_query_heads, w.head_dim), dtype=torch.bfloat16, device=dev)
        got.view(-1).view(torch.uint8).copy_(device_bytes(g.output(step), nbytes, dev))
        torch.cuda.synchronize()
        e = float(np.max(np.abs(got.float().cpu().numpy() - ref)))
        if int(err.item()) != 0 or not status.all() or e >= BF16_ABS:
            msg = f"step {step}: err {int(err.item())} max {e}"
            break
    torch.cuda.synchronize()
    # leave only once every rank is done storing into this GPU's buffers
    with open(os.path.join(tmp, f"done{rank}"), "w") as f:
        f.write("1")
    t0 = time.time()
    while not all(os.path.exists(os.path.join(tmp, f"done{r}")) for r in range(world)) and time.time() - t0 < 120:
        time.sleep(0.05)
    g.close()
    result[rank] = msg


def test_peer_exchange_gives_every_rank_every_head(tmp_path):
    import torch
    import torch.multiprocessing as mp
    world = min(torch.cuda.device_count(), 4)
    if world < 2:
        pytest.skip("needs two GPUs")
    mgr = mp.Manager()
    result = mgr.dict()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_peer_rank_main, args=(r, world, str(tmp_path), result)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:  # host processes only: every GPU wait in the kernels is bounded
        p.kill()
    assert not alive
    assert [result.get(r) for r in range(world)] == ["ok"] * world
