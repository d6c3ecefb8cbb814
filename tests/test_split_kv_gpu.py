"""Split-KV decode of one long sequence: the page list is cut into per-rank
ranges, each range is decoded with lse_out, and the (out, lse) partials are
merged by the LSE-combine kernel.  On one GPU the ranks are emulated (the
merge input is stacked locally, as the NCCL all-gather would deliver it); with
two or more GPUs visible the real path runs as NCCL ranks."""
import math
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _case(dev, L=20000, hq=32, hkv=8, d=128, seed=3):
    g = torch.Generator(device=dev).manual_seed(seed)
    n_pages = math.ceil(L / 16)
    kc = torch.randn(n_pages, 16, hkv, d, generator=g, device=dev).to(torch.bfloat16)
    vc = torch.randn(n_pages, 16, hkv, d, generator=g, device=dev).to(torch.bfloat16)
    q = (torch.randn(1, hq, d, generator=g, device=dev) * 0.5).to(torch.bfloat16)
    return q, kc, vc, n_pages


@pytest.mark.parametrize("world", [2, 3, 8])
def test_split_kv_emulated_ranks(cuda, world):
    from unifiedkv_b200.multi_gpu import local_range_lens, split_pages
    from unifiedkv_b200.page16_native import lse_combine, page16_decode_attention
    L = 20000
    q, kc, vc, n_pages = _case(cuda, L)
    full_lse = torch.empty(1, 32, dtype=torch.float32, device=cuda)
    full = page16_decode_attention(q, kc, vc, torch.arange(n_pages, dtype=torch.int32, device=cuda)[None],
                                   torch.tensor([L], dtype=torch.int32, device=cuda), softmax_scale=128 ** -0.5,
                                   n_rep=4, lse_out=full_lse)
    parts, lses = [], []
    for s, e in split_pages(n_pages, world):
        lse = torch.empty(1, 32, dtype=torch.float32, device=cuda)
        o = page16_decode_attention(q, kc[s:e], vc[s:e], torch.arange(e - s, dtype=torch.int32, device=cuda)[None],
                                    torch.tensor([local_range_lens(L, s, e)], dtype=torch.int32, device=cuda),
                                    softmax_scale=128 ** -0.5, n_rep=4, lse_out=lse)
        parts.append(o.float().reshape(32, 128))
        lses.append(lse.reshape(32))
    merged, mlse = lse_combine(torch.stack(parts), torch.stack(lses), torch.bfloat16, return_lse=True)
    # partials pass through bf16 outputs of each range: allow 2 bf16 ulps of |out| + 2e-3
    diff = (merged.float() - full.float().reshape(32, 128)).abs()
    assert (diff - 2 ** -7 * full.float().reshape(32, 128).abs()).max().item() < 2e-3
    assert (mlse - full_lse.reshape(32)).abs().max().item() < 1e-3


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _nccl_worker(rank, world, port, q_out):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    try:
        from unifiedkv_b200.multi_gpu import local_range_lens, split_kv_decode, split_pages
        from unifiedkv_b200.page16_native import page16_decode_attention
        L = 20000
        q, kc, vc, n_pages = _case(dev, L)  # identical data on every rank (same seed)
        s, e = split_pages(n_pages, world)[rank]
        out = split_kv_decode(q, kc[s:e], vc[s:e], torch.arange(e - s, dtype=torch.int32, device=dev)[None],
                              torch.tensor([local_range_lens(L, s, e)], dtype=torch.int32, device=dev),
                              128 ** -0.5, 4)
        full = page16_decode_attention(q, kc, vc, torch.arange(n_pages, dtype=torch.int32, device=dev)[None],
                                       torch.tensor([L], dtype=torch.int32, device=dev), softmax_scale=128 ** -0.5,
                                       n_rep=4)
        d = (out.float() - full.float()).abs() - 2 ** -8 * full.float().abs()
        q_out.put((rank, float(d.max().item())))
    finally:
        dist.destroy_process_group()


def test_split_kv_nccl_two_ranks(cuda):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    qq = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_nccl_worker, args=(r, 2, port, qq)) for r in range(2)]
    for p in ps:
        p.start()
    res = sorted(qq.get(timeout=300) for _ in range(2))
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert all(err < 2e-3 for _, err in res), res


# ---- NVLink peer-memory exchange (bpkv_split_kv_merge_p2p) ----

def _p2p_call(L, part, lse, bufs, rank, world, out, lse_out, status, max_polls):
    import ctypes
    from unifiedkv_b200 import _lib
    arr = (ctypes.c_void_p * world)(*bufs)
    rc = L.bpkv_split_kv_merge_p2p(part.data_ptr(), lse.data_ptr(), arr, rank, world, int(part.shape[0]),
                                   int(part.shape[1]), max_polls, out.data_ptr(), _lib.ptr(lse_out),
                                   status.data_ptr(), _lib.dtype_code(part.dtype), _lib.stream_ptr(part.device))
    _lib.check(rc, "split_kv_merge_p2p")


def _alloc_buffer(L, nbytes):
    import ctypes
    from unifiedkv_b200 import _lib
    p = ctypes.c_void_p()
    h = ctypes.create_string_buffer(64)
    _lib.check(L.bpkv_peer_buffer_alloc(nbytes, ctypes.byref(p), h), "peer_exchange_alloc")
    return p.value


def test_p2p_merge_single_rank_calls_in_sequence(cuda):
    """world = 1: the exchange degenerates to this rank's own slot; the output is the
    partial itself, over several calls (the call number and parity advance on the device)."""
    from unifiedkv_b200 import _lib
    L = _lib.lib()
    rows, d = 32, 128
    buf = _alloc_buffer(L, L.bpkv_peer_exchange_bytes(1, rows, d))
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    try:
        for it in range(5):
            part = torch.randn(rows, d, device=cuda).to(torch.bfloat16)
            lse = torch.randn(rows, device=cuda)
            out = torch.empty_like(part)
            lse_out = torch.empty(rows, device=cuda)
            _p2p_call(L, part, lse, [buf], 0, 1, out, lse_out, status, 1 << 20)
            torch.cuda.synchronize()
            assert int(status.item()) == 0
            assert torch.equal(out, part)
            assert torch.allclose(lse_out, lse, rtol=0, atol=1e-6)
    finally:
        L.bpkv_peer_buffer_free(buf)


def test_p2p_merge_wait_runs_out_without_fault(cuda):
    """A peer whose partial never arrives: the merge's wait gives up after max_polls,
    reports status 1 and writes NaN rows; the GPU context stays usable.  (The second
    'rank' is a second local buffer that nobody signals: no GPU fault is provoked.)"""
    from unifiedkv_b200 import _lib
    L = _lib.lib()
    rows, d = 8, 64
    nbytes = L.bpkv_peer_exchange_bytes(2, rows, d)
    own, fake_peer = _alloc_buffer(L, nbytes), _alloc_buffer(L, nbytes)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    try:
        part = torch.randn(rows, d, device=cuda)
        lse = torch.zeros(rows, device=cuda)
        out = torch.zeros_like(part)
        _p2p_call(L, part, lse, [own, fake_peer], 0, 2, out, None, status, 2000)
        torch.cuda.synchronize()
        assert int(status.item()) == 1
        assert torch.isnan(out).all()
        assert torch.equal(part + 1, part + 1)  # the context still runs kernels
    finally:
        L.bpkv_peer_buffer_free(own)
        L.bpkv_peer_buffer_free(fake_peer)


def test_p2p_word_format_and_stale_words_one_gpu(cuda):
    """The exchange words on one GPU, with no kernel waiting on another: rank 1 of a
    two-rank group is emulated by writing its words for each call into rank 0's
    buffer (torch ops) before rank 0's call.  A word is {x0, e, x1, e} (two fp32
    values, each beside the call number e; the row's last word holds lse and 0),
    at [e & 1][source rank][row][word].  Checks: the merge equals the log-sum-exp
    merge of both partials; rank 0's own words land in the peer buffer in that
    format; a word left over from call e-2 (same parity) is not taken for call e
    (the wait runs out: status 1, NaN rows) and the next call works again."""
    from unifiedkv_b200 import _lib
    from oracle.page16 import lse_merge_reference
    L = _lib.lib()
    rows, d, world = 16, 128, 2
    Wd = d // 2 + 1
    nbytes = L.bpkv_peer_exchange_bytes(world, rows, d)
    # plain device buffers stand in for the IPC-mapped ones (16-byte aligned, zeroed)
    own = torch.zeros(nbytes // 4, dtype=torch.int32, device=cuda)
    peer = torch.zeros_like(own)
    n_words = 2 * world * rows * Wd * 4
    own_w = own[:n_words].view(2, world, rows, Wd, 4)
    peer_w = peer[:n_words].view(2, world, rows, Wd, 4)
    g = torch.Generator(device=cuda).manual_seed(17)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    for call in (1, 2, 3, 4, 5):
        par = call & 1
        part0 = torch.randn(rows, d, generator=g, device=cuda).to(torch.bfloat16)
        lse0 = torch.randn(rows, generator=g, device=cuda)
        o1 = torch.randn(rows, d, generator=g, device=cuda)
        lse1 = torch.randn(rows, generator=g, device=cuda)
        emulate = call != 4  # call 4: rank 1 "never sends"; its parity slot holds call 2's words
        if emulate:
            vals = torch.cat([o1, torch.stack([lse1, torch.zeros_like(lse1)], 1)], 1).view(rows, Wd, 2)
            own_w[par, 1, :, :, 0] = vals[..., 0].contiguous().view(torch.int32)
            own_w[par, 1, :, :, 2] = vals[..., 1].contiguous().view(torch.int32)
            own_w[par, 1, :, :, 1] = call
            own_w[par, 1, :, :, 3] = call
        out = torch.empty_like(part0)
        lse_out = torch.empty(rows, device=cuda)
        status.zero_()
        _p2p_call(L, part0, lse0, [own.data_ptr(), peer.data_ptr()], 0, world, out, lse_out, status,
                  1 << 20 if emulate else 5000)
        torch.cuda.synchronize()
        # rank 0's words in the peer's buffer, whatever happened to the wait
        pw = peer_w[par, 0]
        assert (pw[..., 1] == call).all() and (pw[..., 3] == call).all()
        sent = torch.stack([pw[..., 0], pw[..., 2]], -1).contiguous().view(torch.float32).view(rows, 2 * Wd)
        assert torch.equal(sent[:, :d], part0.float()) and torch.equal(sent[:, d], lse0)
        if not emulate:
            assert int(status.item()) == 1 and torch.isnan(out.float()).all() and torch.isnan(lse_out).all()
            continue
        assert int(status.item()) == 0
        po = np.stack([part0.float().cpu().numpy(), o1.cpu().numpy()])
        pl = np.stack([lse0.cpu().numpy(), lse1.cpu().numpy()])
        ref_out, ref_lse = lse_merge_reference(po, pl)
        err = np.abs(out.float().cpu().numpy() - ref_out) - 2.0 ** -8 * np.abs(ref_out)
        assert err.max() < 1e-5
        assert np.allclose(lse_out.cpu().numpy(), ref_lse, rtol=0, atol=1e-5)


def _p2p_worker(rank, world, port, q_out):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    try:
        from unifiedkv_b200.multi_gpu import PeerMerge, local_range_lens, split_kv_decode, split_pages
        from unifiedkv_b200.page16_native import page16_decode_attention
        L = 20000
        q, kc, vc, n_pages = _case(dev, L)
        s, e = split_pages(n_pages, world)[rank]
        bt = torch.arange(e - s, dtype=torch.int32, device=dev)[None]
        lens = torch.tensor([local_range_lens(L, s, e)], dtype=torch.int32, device=dev)
        peer = PeerMerge(rows=32, head_dim=128)
        errs = []
        g = torch.Generator(device=dev).manual_seed(11)
        for it in range(4):  # several calls: both parities, call number advancing on the device
            qi = (torch.randn(1, 32, 128, generator=g, device=dev) * 0.5).to(torch.bfloat16)
            out_p2p = split_kv_decode(qi, kc[s:e], vc[s:e], bt, lens, 128 ** -0.5, 4, peer=peer)
            out_nccl = split_kv_decode(qi, kc[s:e], vc[s:e], bt, lens, 128 ** -0.5, 4)
            full = page16_decode_attention(qi, kc, vc, torch.arange(n_pages, dtype=torch.int32, device=dev)[None],
                                           torch.tensor([L], dtype=torch.int32, device=dev),
                                           softmax_scale=128 ** -0.5, n_rep=4)
            peer.check()
            errs.append(float(((out_p2p.float() - full.float()).abs() - 2 ** -8 * full.float().abs()).max().item()))
            errs.append(float((out_p2p.float() - out_nccl.float()).abs().max().item()))
        peer.close()
        q_out.put((rank, max(errs)))
    finally:
        dist.destroy_process_group()


def test_split_kv_p2p_two_ranks(cuda):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    qq = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_p2p_worker, args=(r, 2, port, qq)) for r in range(2)]
    for p in ps:
        p.start()
    res = sorted(qq.get(timeout=300) for _ in range(2))
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert all(err < 2e-3 for _, err in res), res
