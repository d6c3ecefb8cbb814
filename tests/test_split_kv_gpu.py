"""Split-KV decode of one long sequence: the page list is cut into per-rank
ranges, each range is decoded into fp32 partials, and the (out, lse) partials
are merged by log-sum-exp.  Every result is compared with the fp64 oracle of
the WHOLE sequence (oracle.page16, the reference's gather-then-attention path)
at max-abs 2e-3, with no allowance for rounded partials: partials stay fp32
until the final merge.  On one GPU the ranks are emulated (the merge input is
stacked locally, or the peer's exchange words are written by torch ops); with
two or more GPUs visible the real path also runs as NCCL ranks."""
import ctypes
import math
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

TOL = 2e-3  # max-abs against the fp64 oracle (bf16 inputs)


def _case(dev, L=20000, hq=32, hkv=8, d=128, seed=3):
    g = torch.Generator(device=dev).manual_seed(seed)
    n_pages = math.ceil(L / 16)
    kc = torch.randn(n_pages, 16, hkv, d, generator=g, device=dev).to(torch.bfloat16)
    vc = torch.randn(n_pages, 16, hkv, d, generator=g, device=dev).to(torch.bfloat16)
    q = (torch.randn(1, hq, d, generator=g, device=dev) * 0.5).to(torch.bfloat16)
    return q, kc, vc, n_pages


def _oracle(q, kc, vc, L, n_rep=4):
    from oracle.page16 import page16_decode_reference
    n_pages = kc.shape[0]
    out, lse = page16_decode_reference(q.float().cpu().numpy(), kc.float().cpu().numpy(), vc.float().cpu().numpy(),
                                       np.arange(n_pages, dtype=np.int32)[None], np.array([L], np.int32),
                                       q.shape[-1] ** -0.5, n_rep, return_lse=True)
    return out, lse


def _range_args(dev, L, s, e):
    from unifiedkv_b200.multi_gpu import local_range_lens
    return (torch.arange(e - s, dtype=torch.int32, device=dev)[None],
            torch.tensor([local_range_lens(L, s, e)], dtype=torch.int32, device=dev))


@pytest.mark.parametrize("world", [2, 3, 8])
def test_split_kv_emulated_ranks_fp32_partials(cuda, world):
    from unifiedkv_b200.multi_gpu import decode_partial, split_pages
    from unifiedkv_b200.page16_native import lse_combine
    L = 20000
    q, kc, vc, n_pages = _case(cuda, L)
    ref, ref_lse = _oracle(q, kc, vc, L)
    parts, lses = [], []
    for s, e in split_pages(n_pages, world):
        bt, ln = _range_args(cuda, L, s, e)
        o, lse = decode_partial(q, kc[s:e], vc[s:e], bt, ln, 128 ** -0.5, 4)
        assert o.dtype == torch.float32
        parts.append(o.reshape(32, 128))
        lses.append(lse.reshape(32))
    merged, mlse = lse_combine(torch.stack(parts), torch.stack(lses), torch.float32, return_lse=True)
    assert np.abs(merged.cpu().numpy() - ref[0]).max() < 1e-4  # fp32 end to end
    merged16 = lse_combine(torch.stack(parts), torch.stack(lses), torch.bfloat16)
    assert np.abs(merged16.float().cpu().numpy() - ref[0]).max() < TOL
    assert np.abs(mlse.cpu().numpy() - ref_lse[0]).max() < 1e-3


@pytest.mark.parametrize("num_splits", [0, 1, 7, 64, 296])
def test_fused_split_decode_one_rank(cuda, num_splits):
    """world = 1: decode partials + the fused combine (no exchange) equal the oracle;
    any split count (1 CTA to 2 per SM) gives the same answer."""
    from unifiedkv_b200.multi_gpu import _split_decode
    L = 20000
    q, kc, vc, n_pages = _case(cuda, L, seed=5)
    ref, ref_lse = _oracle(q, kc, vc, L)
    bt, ln = _range_args(cuda, L, 0, n_pages)
    lse = torch.empty(1, 32, device=cuda)
    out = _split_decode(q, kc, vc, bt, ln, 128 ** -0.5, 4, out_dtype=torch.bfloat16, lse_out=lse,
                        num_splits=num_splits)
    out32 = _split_decode(q, kc, vc, bt, ln, 128 ** -0.5, 4, out_dtype=torch.float32, num_splits=num_splits)
    torch.cuda.synchronize()
    assert np.abs(out.float().cpu().numpy() - ref).max() < TOL
    assert np.abs(out32.cpu().numpy() - ref).max() < 1e-4
    assert np.abs(lse.cpu().numpy() - ref_lse).max() < 1e-3


@pytest.mark.parametrize("hkv,d,dtype", [(8, 64, torch.bfloat16), (4, 256, torch.bfloat16), (8, 128, torch.float16),
                                         (2, 96, torch.bfloat16)])
def test_fused_split_decode_head_dims(cuda, hkv, d, dtype):
    """The fused kernel's 32-column chunks and word ranges for other head sizes (96: the
    last chunk is partial and the generic decode kernel produces the partials)."""
    from oracle.page16 import page16_decode_reference
    from tests.golden.inputs import page16_case
    from unifiedkv_b200.multi_gpu import _split_decode
    hq = 4 * hkv
    q, k, v, bt, lens = page16_case(seed=d, batch=2, hq=hq, hkv=hkv, d=d, lens=(3000, 77), num_pages=260,
                                    scale_std=0.5)
    t = [torch.from_numpy(x).to(cuda, dtype) for x in (q, k, v)]
    lse = torch.empty(2, hq, device=cuda)
    out = _split_decode(t[0], t[1], t[2], torch.from_numpy(bt).to(cuda), torch.from_numpy(lens).to(cuda),
                        d ** -0.5, 4, out_dtype=torch.float32, lse_out=lse)
    torch.cuda.synchronize()
    ref, ref_lse = page16_decode_reference(*(x.float().cpu().numpy() for x in t), bt, lens, d ** -0.5, 4,
                                           return_lse=True)
    assert np.abs(out.cpu().numpy() - ref).max() < 1e-4
    assert np.abs(lse.cpu().numpy() - ref_lse).max() < 1e-3


def test_fused_split_decode_batch_and_empty_rows(cuda):
    """Several requests in one call, one of them without tokens in this range
    (NaN row, lse -inf: the reference's 0/0), with ragged lengths."""
    from oracle.page16 import page16_decode_reference
    from tests.golden.inputs import page16_case
    from unifiedkv_b200.multi_gpu import _split_decode
    q, k, v, bt, lens = page16_case(seed=9, batch=4, hq=16, hkv=4, d=128, lens=(0, 17, 300, 2000), num_pages=256,
                                    scale_std=0.5)
    t = [torch.from_numpy(x).to(cuda, torch.bfloat16) for x in (q, k, v)]
    lse = torch.empty(4, 16, device=cuda)
    out = _split_decode(t[0], t[1], t[2], torch.from_numpy(bt).to(cuda), torch.from_numpy(lens).to(cuda),
                        128 ** -0.5, 4, out_dtype=torch.bfloat16, lse_out=lse)
    torch.cuda.synchronize()
    ref = page16_decode_reference(*(x.float().cpu().numpy() for x in t), bt, lens, 128 ** -0.5, 4)
    o = out.float().cpu().numpy()
    assert np.isnan(o[0]).all() and np.isneginf(lse[0].cpu().numpy()).all()
    assert np.abs(o[1:] - ref[1:]).max() < TOL


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
        from unifiedkv_b200.multi_gpu import split_kv_decode, split_pages
        L = 20000
        q, kc, vc, n_pages = _case(dev, L)  # identical data on every rank (same seed)
        s, e = split_pages(n_pages, world)[rank]
        bt, ln = _range_args(dev, L, s, e)
        out = split_kv_decode(q, kc[s:e], vc[s:e], bt, ln, 128 ** -0.5, 4)
        ref, _ = _oracle(q, kc, vc, L)
        q_out.put((rank, float(np.abs(out.float().cpu().numpy() - ref).max())))
    finally:
        dist.destroy_process_group()


def _run_two_ranks(target):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    qq = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=target, args=(r, 2, port, qq)) for r in range(2)]
    for p in ps:
        p.start()
    res = sorted(qq.get(timeout=300) for _ in range(2))
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    return res


def test_split_kv_nccl_two_ranks(cuda):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    res = _run_two_ranks(_nccl_worker)
    assert all(err < TOL for _, err in res), res


# ---- NVLink peer-memory exchange ----

def _p2p_call(L, part, lse, bufs, rank, world, out, lse_out, status, max_polls):
    from unifiedkv_b200 import _lib
    arr = (ctypes.c_void_p * world)(*bufs)
    rc = L.bpkv_split_kv_merge_p2p(part.data_ptr(), lse.data_ptr(), arr, rank, world, int(part.shape[0]),
                                   int(part.shape[1]), max_polls, out.data_ptr(), _lib.ptr(lse_out),
                                   status.data_ptr(), _lib.dtype_code(part.dtype), _lib.dtype_code(out.dtype),
                                   _lib.stream_ptr(part.device))
    _lib.check(rc, "split_kv_merge_p2p")


def _alloc_buffer(L, nbytes):
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


def _word_views(nbytes, world, rows, d, dev):
    """Plain device buffers standing in for the IPC-mapped ones (16-byte aligned, zeroed),
    viewed as [parity][source rank][row][word][4 x u32]; a word is two 64-bit halves,
    each (fp32 value bits) | (call number << 32), i.e. u32 {x0, e, x1, e}."""
    Wd = d // 2 + 1
    own = torch.zeros(nbytes // 4, dtype=torch.int32, device=dev)
    peer = torch.zeros_like(own)
    n = 2 * world * rows * Wd * 4
    return own, peer, own[:n].view(2, world, rows, Wd, 4), peer[:n].view(2, world, rows, Wd, 4)


def _write_words(words, par, src, o, lse, call):
    rows, d = o.shape
    Wd = d // 2 + 1
    vals = torch.cat([o.float(), torch.stack([lse.float(), torch.zeros_like(lse.float())], 1)], 1).view(rows, Wd, 2)
    words[par, src, :, :, 0] = vals[..., 0].contiguous().view(torch.int32)
    words[par, src, :, :, 2] = vals[..., 1].contiguous().view(torch.int32)
    words[par, src, :, :, 1] = call
    words[par, src, :, :, 3] = call


def _read_words(words, par, src, d):
    rows = words.shape[2]
    Wd = d // 2 + 1
    pw = words[par, src]
    vals = torch.stack([pw[..., 0], pw[..., 2]], -1).contiguous().view(torch.float32).view(rows, 2 * Wd)
    return pw, vals[:, :d], vals[:, d]


def test_p2p_word_format_and_stale_words_one_gpu(cuda):
    """The exchange words on one GPU, with no kernel waiting on another: rank 1 of a
    two-rank group is emulated by writing its words for each call into rank 0's
    buffer (torch ops) before rank 0's call.  Checks: the merge equals the
    log-sum-exp merge of both partials; rank 0's own words land in the peer buffer
    in that format; a word left over from call e-2 (same parity) is not taken for
    call e (the wait runs out: status 1, NaN rows) and the next call works again.
    The partial is fp32 and the output bf16 (partial and output types differ)."""
    from unifiedkv_b200 import _lib
    from oracle.page16 import lse_merge_reference
    L = _lib.lib()
    rows, d, world = 16, 128, 2
    nbytes = L.bpkv_peer_exchange_bytes(world, rows, d)
    own, peer, own_w, peer_w = _word_views(nbytes, world, rows, d, cuda)
    g = torch.Generator(device=cuda).manual_seed(17)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    for call in (1, 2, 3, 4, 5):
        par = call & 1
        part0 = torch.randn(rows, d, generator=g, device=cuda)
        lse0 = torch.randn(rows, generator=g, device=cuda)
        o1 = torch.randn(rows, d, generator=g, device=cuda)
        lse1 = torch.randn(rows, generator=g, device=cuda)
        emulate = call != 4  # call 4: rank 1 "never sends"; its parity slot holds call 2's words
        if emulate:
            _write_words(own_w, par, 1, o1, lse1, call)
        out = torch.empty(rows, d, dtype=torch.bfloat16, device=cuda)
        lse_out = torch.empty(rows, device=cuda)
        status.zero_()
        _p2p_call(L, part0, lse0, [own.data_ptr(), peer.data_ptr()], 0, world, out, lse_out, status,
                  1 << 20 if emulate else 5000)
        torch.cuda.synchronize()
        pw, sent_o, sent_l = _read_words(peer_w, par, 0, d)
        assert (pw[..., 1] == call).all() and (pw[..., 3] == call).all()
        assert torch.equal(sent_o, part0) and torch.equal(sent_l, lse0)
        if not emulate:
            assert int(status.item()) == 1 and torch.isnan(out.float()).all() and torch.isnan(lse_out).all()
            continue
        assert int(status.item()) == 0
        ref_out, ref_lse = lse_merge_reference(np.stack([part0.cpu().numpy(), o1.cpu().numpy()]),
                                               np.stack([lse0.cpu().numpy(), lse1.cpu().numpy()]))
        assert np.abs(out.float().cpu().numpy() - ref_out).max() < 2 ** -8 * max(1.0, np.abs(ref_out).max())
        assert np.allclose(lse_out.cpu().numpy(), ref_lse, rtol=0, atol=1e-5)


def test_fused_split_decode_emulated_peer_one_gpu(cuda):
    """bpkv_split_kv_decode_p2p as rank 0 of 2 on one GPU: rank 1's fp32 partial of
    the second half of the pages is written into rank 0's buffer as words (torch
    ops) before each call.  The merged output matches the fp64 oracle of the whole
    sequence; rank 0's words in the peer's buffer carry exactly its fp32 local
    combine (the world = 1 result of the same kernel) and the call number; a stale
    same-parity word is not taken (status 1, NaN rows, then the next call works)."""
    from unifiedkv_b200 import _lib
    from unifiedkv_b200.multi_gpu import _split_decode, decode_partial, split_pages
    Lb = _lib.lib()
    L, world, rows, d = 20000, 2, 32, 128
    q, kc, vc, n_pages = _case(cuda, L, seed=21)
    (s0, e0), (s1, e1) = split_pages(n_pages, world)
    bt0, ln0 = _range_args(cuda, L, s0, e0)
    bt1, ln1 = _range_args(cuda, L, s1, e1)
    nbytes = Lb.bpkv_peer_exchange_bytes(world, rows, d)
    own, peer, own_w, peer_w = _word_views(nbytes, world, rows, d, cuda)
    bufs = (ctypes.c_void_p * world)(own.data_ptr(), peer.data_ptr())
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    g = torch.Generator(device=cuda).manual_seed(5)
    for call in (1, 2, 3, 4, 5):
        par = call & 1
        qi = (torch.randn(1, 32, 128, generator=g, device=cuda) * 0.5).to(torch.bfloat16)
        emulate = call != 4
        o1, l1 = decode_partial(qi, kc[s1:e1], vc[s1:e1], bt1, ln1, 128 ** -0.5, 4)
        if emulate:
            _write_words(own_w, par, 1, o1.reshape(rows, d), l1.reshape(rows), call)
        o0, l0 = decode_partial(qi, kc[s0:e0], vc[s0:e0], bt0, ln0, 128 ** -0.5, 4)
        status.zero_()
        lse = torch.empty(1, 32, device=cuda)
        out = _split_decode(qi, kc[s0:e0], vc[s0:e0], bt0, ln0, 128 ** -0.5, 4, out_dtype=torch.bfloat16,
                            lse_out=lse, bufs=bufs, rank=0, world=world,
                            max_polls=(1 << 20) if emulate else 5000, status=status)
        torch.cuda.synchronize()
        pw, sent_o, sent_l = _read_words(peer_w, par, 0, d)
        assert (pw[..., 1] == call).all() and (pw[..., 3] == call).all()
        assert torch.equal(sent_o, o0.reshape(rows, d)) and torch.equal(sent_l, l0.reshape(rows))
        if not emulate:
            assert int(status.item()) == 1 and torch.isnan(out.float()).all()
            continue
        assert int(status.item()) == 0
        ref, ref_lse = _oracle(qi, kc, vc, L)
        assert np.abs(out.float().cpu().numpy() - ref).max() < TOL
        assert np.abs(lse.cpu().numpy() - ref_lse).max() < 1e-3


def _p2p_worker(rank, world, port, q_out):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    try:
        from unifiedkv_b200.multi_gpu import PeerMerge, split_kv_decode, split_pages
        L = 20000
        q, kc, vc, n_pages = _case(dev, L)
        s, e = split_pages(n_pages, world)[rank]
        bt, ln = _range_args(dev, L, s, e)
        peer = PeerMerge(rows=32, head_dim=128)
        errs = []
        g = torch.Generator(device=dev).manual_seed(11)
        for it in range(4):  # several calls: both parities, call number advancing on the device
            qi = (torch.randn(1, 32, 128, generator=g, device=dev) * 0.5).to(torch.bfloat16)
            out_p2p = split_kv_decode(qi, kc[s:e], vc[s:e], bt, ln, 128 ** -0.5, 4, peer=peer)
            out_nccl = split_kv_decode(qi, kc[s:e], vc[s:e], bt, ln, 128 ** -0.5, 4)
            peer.check()
            ref, _ = _oracle(qi, kc, vc, L)
            errs.append(float(np.abs(out_p2p.float().cpu().numpy() - ref).max()))
            errs.append(float(np.abs(out_nccl.float().cpu().numpy() - ref).max()))
        peer.close()
        q_out.put((rank, max(errs)))
    finally:
        dist.destroy_process_group()


def test_split_kv_p2p_two_ranks(cuda):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    res = _run_two_ranks(_p2p_worker)
    assert all(err < TOL for _, err in res), res
