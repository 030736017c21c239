"""Block movers on the GPU against the oracle: batched copy-on-write copies,
swap gather/scatter round trips and the KV append, all bit-exact."""
import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu


def _dev():
    import torch
    return torch.device("cuda", 0)


def _stream():
    import torch
    return torch.cuda.current_stream().cuda_stream


def test_copy_blocks_matches_the_oracle_bit_for_bit():
    import torch

    import qvp
    stride, nblk = 32768, 64
    rng = np.random.default_rng(0)
    host = rng.integers(0, 256, size=stride * nblk, dtype=np.uint8)
    pool = torch.from_numpy(host.copy()).to(_dev())
    src = rng.permutation(nblk)[:20]
    dst = rng.permutation([i for i in range(nblk) if i not in set(src)])[:20]
    pairs = np.stack([src, dst], 1).reshape(-1).astype(np.int32)
    pairs_d = torch.from_numpy(pairs).to(_dev())
    err = torch.zeros(1, dtype=torch.int32, device=_dev())
    st = qvp.lib.qvp_copy_blocks(pool.data_ptr(), stride, nblk, stride, pairs_d.data_ptr(), 20, err.data_ptr(),
                                 _stream())
    assert st == 0
    torch.cuda.synchronize()
    oracle.port_copy_blocks(host, stride, nblk, stride, pairs)
    assert np.array_equal(pool.cpu().numpy(), host)
    assert err.item() == 0


@pytest.mark.parametrize("nbytes", [65536, 256, 4096 + 48, 100])
def test_gather_scatter_round_trip_through_pinned_host_memory(nbytes):
    import torch

    import qvp
    stride, nblk = max(256, (nbytes + 255) // 256 * 256), 40
    rng = np.random.default_rng(nbytes)
    host = rng.integers(0, 256, size=stride * nblk, dtype=np.uint8)
    pool = torch.from_numpy(host).to(_dev())
    ids = rng.permutation(nblk)[:17].astype(np.int32)
    ids_d = torch.from_numpy(ids).to(_dev())
    err = torch.zeros(1, dtype=torch.int32, device=_dev())
    for staging in (torch.empty(17 * nbytes, dtype=torch.uint8, device=_dev()),
                    torch.empty(17 * nbytes, dtype=torch.uint8).pin_memory()):
        assert qvp.lib.qvp_gather_blocks(pool.data_ptr(), stride, nblk, nbytes, ids_d.data_ptr(), 17,
                                         staging.data_ptr(), err.data_ptr(), _stream()) == 0
        torch.cuda.synchronize()
        got = staging.cpu().numpy().reshape(17, nbytes)
        want = host.reshape(nblk, stride)[ids, :nbytes]
        assert np.array_equal(got, want)
        # scatter into other blocks, then compare bytes
        dst = np.array([i for i in range(nblk) if i not in set(ids)][:17], dtype=np.int32)
        dst_d = torch.from_numpy(dst).to(_dev())
        assert qvp.lib.qvp_scatter_blocks(pool.data_ptr(), stride, nblk, nbytes, dst_d.data_ptr(), 17,
                                          staging.data_ptr(), err.data_ptr(), _stream()) == 0
        torch.cuda.synchronize()
        now = pool.cpu().numpy().reshape(nblk, stride)
        assert np.array_equal(now[dst, :nbytes], want)
        pool.copy_(torch.from_numpy(host))
    assert err.item() == 0


def test_movers_flag_bad_ids_and_skip_them():
    import torch

    import qvp
    pool = torch.zeros(4 * 256, dtype=torch.uint8, device=_dev())
    pairs = torch.tensor([0, 7, -1, 1], dtype=torch.int32, device=_dev())
    err = torch.zeros(1, dtype=torch.int32, device=_dev())
    assert qvp.lib.qvp_copy_blocks(pool.data_ptr(), 256, 4, 256, pairs.data_ptr(), 2, err.data_ptr(), _stream()) == 0
    torch.cuda.synchronize()
    assert err.item() & qvp.DEVERR_BAD_BLOCK
    assert int(pool.sum()) == 0


def test_kv_append_writes_the_new_token_rows():
    import torch

    import qvp
    T, L, H, D, elem = 16, 2, 4, 128, 2
    shape = qvp.make_shape(T, L, H, D, elem)
    stride = qvp.block_stride(shape)
    nblk, B, pitch = 32, 5, 4
    pool = torch.zeros(nblk * stride, dtype=torch.uint8, device=_dev())
    rng = np.random.default_rng(3)
    tables = rng.permutation(nblk)[:B * pitch].reshape(B, pitch).astype(np.int32)
    pos = rng.integers(0, pitch * T, size=B).astype(np.int32)
    k = rng.integers(0, 256, size=B * H * D * elem, dtype=np.uint8)
    v = rng.integers(0, 256, size=B * H * D * elem, dtype=np.uint8)
    err = torch.zeros(1, dtype=torch.int32, device=_dev())
    td, pd = torch.from_numpy(tables).to(_dev()), torch.from_numpy(pos).to(_dev())
    kd, vd = torch.from_numpy(k).to(_dev()), torch.from_numpy(v).to(_dev())
    import ctypes as C
    assert qvp.lib.qvp_kv_append(pool.data_ptr(), stride, nblk, C.byref(shape), 1, B, pitch, td.data_ptr(),
                                 pd.data_ptr(), kd.data_ptr(), vd.data_ptr(), err.data_ptr(), _stream()) == 0
    torch.cuda.synchronize()
    got = pool.cpu().numpy().reshape(nblk, stride)
    row = H * D * elem
    expect = np.zeros((nblk, stride), dtype=np.uint8)
    for b in range(B):
        blk = tables[b, pos[b] // T]
        base = (1 * 2 * T + pos[b] % T) * row  # layer 1, K stream
        expect[blk, base:base + row] = k[b * row:(b + 1) * row]
        base += T * row  # V stream
        expect[blk, base:base + row] = v[b * row:(b + 1) * row]
    assert np.array_equal(got, expect)
    assert err.item() == 0


def test_fetch_host_copies_pinned_bytes_at_any_alignment():
    import torch

    import qvp
    rng = np.random.default_rng(4)
    src = torch.from_numpy(rng.integers(0, 256, size=(3 << 20) + 64, dtype=np.uint8)).pin_memory()
    dst = torch.zeros_like(src, device=_dev())
    for off_s, off_d, n in ((0, 0, 0), (0, 0, 1), (3, 5, 17), (16, 32, 4096), (1, 0, (1 << 20) + 3),
                            (0, 16, 3 << 20)):
        dst.zero_()
        assert qvp.lib.qvp_fetch_host(dst.data_ptr() + off_d, src.data_ptr() + off_s, n, _stream()) == 0
        torch.cuda.synchronize()
        got = dst.cpu().numpy()
        assert np.array_equal(got[off_d:off_d + n], src.numpy()[off_s:off_s + n])
        assert not got[:off_d].any() and not got[off_d + n:].any()
    assert qvp.lib.qvp_fetch_host(None, src.data_ptr(), 16, _stream()) != 0
