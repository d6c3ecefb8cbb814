"""Stream and CUDA-graph behaviour of the library calls.

Every entry point launches on the caller's current stream, as the reference's
Triton launches do (core/page16_native.py:83-150), and never synchronises with
the host.  So a call can run on a side stream, and a sequence of calls can be
captured into a CUDA graph; the decode bench replays a graph of the 32-layer
step, and the compression chain's launches are programmatic dependent launches,
which a capture turns into programmatic graph edges.  Each test checks two
things.  A side-stream call and a graph replay give the same bits as the eager
call on the default stream.  A replay after new values were written into the
captured input buffers (new queries, lengths, block tables, keys) computes on
those values, checked against the eager call and, for decode, against the
oracle within the 2e-3 bar.
"""
import math

import numpy as np
import pytest
import torch

from oracle.page16 import page16_decode_reference
from tests.golden.inputs import compress_case, page16_case

pytestmark = pytest.mark.gpu


def _side_stream(cuda, fn):
    cur = torch.cuda.current_stream(cuda)
    s = torch.cuda.Stream(cuda)
    s.wait_stream(cur)
    with torch.cuda.stream(s):
        out = fn()
    cur.wait_stream(s)
    return out


def _capture(cuda, fn):
    """Warm up on a side stream (as torch recommends), then capture ``fn``."""
    _side_stream(cuda, fn)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out = fn()
    return g, out


def _err(out, ref):
    ref = np.asarray(ref, np.float64)
    return float(np.nanmax(np.abs(out - ref) - 2.0 ** -8 * np.abs(ref)))


def test_decode_side_stream_and_graph_replay(cuda):
    from unifiedkv_b200.page16_native import page16_decode_attention
    hq, hkv, d, dtype = 32, 8, 128, torch.bfloat16
    lens0 = (1, 16, 300, 2049, 4096, 77)
    q, k, v, bt, lens = page16_case(seed=61, batch=len(lens0), hq=hq, hkv=hkv, d=d, lens=lens0,
                                    num_pages=1200, max_blocks=256, scale_std=0.5)
    tk = torch.from_numpy(k).to(cuda, dtype)
    tv = torch.from_numpy(v).to(cuda, dtype)
    sq = torch.from_numpy(q).to(cuda, dtype)
    sbt = torch.from_numpy(bt).to(cuda)
    sl = torch.from_numpy(lens).to(cuda)
    slse = torch.empty(len(lens0), hq, device=cuda)

    def step():
        return page16_decode_attention(sq, tk, tv, sbt, sl, softmax_scale=d ** -0.5, n_rep=hq // hkv,
                                       lse_out=slse)

    eager = step().clone()
    lse_eager = slse.clone()
    side = _side_stream(cuda, step)
    torch.cuda.synchronize()
    assert torch.equal(side, eager) and torch.equal(slse, lse_eager)

    g, gout = _capture(cuda, step)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(gout, eager) and torch.equal(slse, lse_eager)

    # new queries, lengths and block tables in the captured buffers
    q2, _, _, bt2, lens2 = page16_case(seed=62, batch=len(lens0), hq=hq, hkv=hkv, d=d,
                                       lens=(4000, 0, 15, 33, 1, 2500), num_pages=1200, max_blocks=256,
                                       scale_std=0.5)
    sq.copy_(torch.from_numpy(q2).to(cuda, dtype))
    sbt.copy_(torch.from_numpy(bt2).to(cuda))
    sl.copy_(torch.from_numpy(lens2).to(cuda))
    g.replay()
    torch.cuda.synchronize()
    replayed, lse_replayed = gout.clone(), slse.clone()
    eager2 = step()
    torch.cuda.synchronize()
    torch.testing.assert_close(replayed, eager2, rtol=0, atol=0, equal_nan=True)
    torch.testing.assert_close(lse_replayed, slse, rtol=0, atol=0, equal_nan=True)
    ref = page16_decode_reference(sq.float().cpu().numpy(), tk.float().cpu().numpy(), tv.float().cpu().numpy(),
                                  bt2, lens2, d ** -0.5, hq // hkv)
    live = lens2 > 0
    assert _err(replayed.float().cpu().numpy()[live], ref[live]) < 2e-3
    assert torch.isnan(replayed[~torch.from_numpy(live).to(cuda)].float()).all()  # 0/0 row, as in the reference


def test_fused_append_decode_loop_in_a_graph(cuda):
    """The decode loop pattern: one captured step (append this token, attend)
    replayed while the lengths advance in place; pools and outputs stay
    bit-identical to the eager loop."""
    from unifiedkv_b200.page16_native import page16_decode_attention
    hq, hkv, d, dtype = 16, 4, 128, torch.bfloat16
    lens0, n_steps = (15, 16, 31, 500), 4
    # pages for the final lengths: an append must never land in a 0-padded table slot (page 0 is
    # shared padding, so several requests would store into it); the scheduler allocates first too
    q, k, v, bt, _ = page16_case(seed=63, batch=4, hq=hq, hkv=hkv, d=d, lens=tuple(l + n_steps for l in lens0),
                                 num_pages=200, max_blocks=40, scale_std=0.5)
    lens = np.asarray(lens0, np.int32)
    k0 = torch.from_numpy(k).to(cuda, dtype)
    v0 = torch.from_numpy(v).to(cuda, dtype)
    kg, vg, ke, ve = k0.clone(), v0.clone(), k0.clone(), v0.clone()
    sbt = torch.from_numpy(bt).to(cuda)
    gen = torch.Generator(device="cpu").manual_seed(5)
    steps = [(torch.randn(4, hq, d, generator=gen), torch.randn(4, hkv, d, generator=gen),
              torch.randn(4, hkv, d, generator=gen)) for _ in range(n_steps)]
    sq = torch.zeros(4, hq, d, device=cuda, dtype=dtype)
    skn = torch.zeros(4, hkv, d, device=cuda, dtype=dtype)
    svn = torch.zeros_like(skn)
    lens_g = torch.from_numpy(lens).to(cuda) + 1  # lengths include the token being appended
    lens_e = lens_g.clone()

    def step(kc, vc, lens_t):
        return page16_decode_attention(sq, kc, vc, sbt, lens_t, softmax_scale=d ** -0.5, n_rep=hq // hkv,
                                       k_new=skn, v_new=svn)

    g, gout = _capture(cuda, lambda: step(kg, vg, lens_g))
    # warm-up and capture appended zeros into kg/vg: start the replayed pool from the original again
    kg.copy_(k0)
    vg.copy_(v0)
    for qn, kn, vn in steps:
        sq.copy_(qn.to(cuda, dtype))
        skn.copy_(kn.to(cuda, dtype))
        svn.copy_(vn.to(cuda, dtype))
        g.replay()
        out_e = step(ke, ve, lens_e)
        torch.cuda.synchronize()
        assert torch.equal(gout, out_e)
        assert torch.equal(kg, ke) and torch.equal(vg, ve)
        lens_g += 1
        lens_e += 1
    # every appended token sits at its position in the pool
    for b, l0 in enumerate(lens0):
        for t, (_, kn, _) in enumerate(steps):
            pos = l0 + t
            assert torch.equal(ke[bt[b, pos // 16], pos % 16], kn[b].to(cuda, dtype))


def test_compression_chain_in_a_graph(cuda):
    """Scores -> top-k -> compaction (five programmatic dependent launches)
    captured once; replays on new keys match the eager chain bit for bit."""
    from unifiedkv_b200.compress import SMOOTH_ALWAYS, block_scores, topk_blocks
    from unifiedkv_b200.pool import write_pages
    dtype, sink, obs, L, h_kv, d = torch.bfloat16, 64, 64, 4100, 8, 128
    K, V, Q, _ = compress_case(seed=71, h_kv=h_kv, L=L, d=d, n_rep=4, window=obs)
    tk = torch.from_numpy(np.asarray(K, np.float32)).to(cuda, dtype)
    tv = torch.from_numpy(np.asarray(V, np.float32)).to(cuda, dtype)
    tq = torch.from_numpy(np.asarray(Q, np.float32)).to(cuda, dtype)
    n = math.ceil((L - sink - obs) / 16)
    k_blocks = n // 4
    eff_pages = math.ceil((sink + 16 * k_blocks + obs) / 16)
    dst = torch.randperm(400, generator=torch.Generator().manual_seed(3))[:eff_pages].to(cuda, torch.int32)

    def chain(kp, vp):
        s = block_scores(tk, tq, sink, obs, smooth=SMOOTH_ALWAYS)
        sel = topk_blocks(s, k_blocks)
        write_pages(kp, vp, tk, tv, dst, sel, k_blocks, sink, obs)
        return s, sel

    def pools():
        return (torch.zeros(400, 16, h_kv, d, device=cuda, dtype=dtype),
                torch.zeros(400, 16, h_kv, d, device=cuda, dtype=dtype))

    ke, ve = pools()
    s_e, sel_e = chain(ke, ve)
    s_e, sel_e = s_e.clone(), sel_e.clone()
    ks, vs = pools()
    s_s, sel_s = _side_stream(cuda, lambda: chain(ks, vs))
    torch.cuda.synchronize()
    assert torch.equal(s_s, s_e) and torch.equal(sel_s, sel_e)
    assert torch.equal(ks, ke) and torch.equal(vs, ve)

    kg, vg = pools()
    g, (s_g, sel_g) = _capture(cuda, lambda: chain(kg, vg))
    kg.zero_()
    vg.zero_()
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(s_g, s_e) and torch.equal(sel_g, sel_e)
    assert torch.equal(kg, ke) and torch.equal(vg, ve)

    # new keys and values: the replay selects and compacts from them
    K2, V2, _, _ = compress_case(seed=72, h_kv=h_kv, L=L, d=d, n_rep=4, window=obs, hot_blocks=16, sink=sink)
    tk.copy_(torch.from_numpy(np.asarray(K2, np.float32)).to(cuda, dtype))
    tv.copy_(torch.from_numpy(np.asarray(V2, np.float32)).to(cuda, dtype))
    g.replay()
    torch.cuda.synchronize()
    s_r, sel_r = s_g.clone(), sel_g.clone()
    k2, v2 = pools()
    s_e2, sel_e2 = chain(k2, v2)
    torch.cuda.synchronize()
    assert not torch.equal(sel_r, sel_e)  # the hot blocks moved the selection
    assert torch.equal(s_r, s_e2) and torch.equal(sel_r, sel_e2)
    assert torch.equal(kg, k2) and torch.equal(vg, v2)


def test_paged_prefill_side_stream_and_graph(cuda):
    """Chunked prefill over paged past with device-side lengths (the capture
    form of the call): side stream and graph replays match eager bits, also
    after the lengths and queries in the captured buffers change."""
    from unifiedkv_b200.chunked_prefill import paged_chunk_prefill
    from oracle.prefill import chunk_attention
    hq, hkv, d, dtype = 32, 8, 128, torch.bfloat16
    past, chunk = [0, 100, 3000], [256, 256, 129]
    B, max_q = len(past), max(chunk)
    need = [math.ceil((p + c) / 16) for p, c in zip(past, chunk)]
    n_pages = sum(need) + 8
    gen = torch.Generator(device=cuda).manual_seed(9)
    kc = torch.randn(n_pages, 16, hkv, d, generator=gen, device=cuda).to(dtype)
    vc = torch.randn(n_pages, 16, hkv, d, generator=gen, device=cuda).to(dtype)
    perm = np.random.default_rng(4).permutation(n_pages)
    bt = np.zeros((B, max(need)), np.int32)
    off = 0
    for b in range(B):
        bt[b, :need[b]] = perm[off:off + need[b]]
        off += need[b]
    sbt = torch.from_numpy(bt).to(cuda)
    sq = torch.randn(sum(chunk), hq, d, generator=gen, device=cuda).to(dtype)
    cu = torch.tensor(np.concatenate([[0], np.cumsum(chunk)]), dtype=torch.int32, device=cuda)
    sk = torch.tensor([p + c for p, c in zip(past, chunk)], dtype=torch.int32, device=cuda)

    def call():
        return paged_chunk_prefill(sq, kc, vc, sbt, None, None, d ** -0.5, hq // hkv, cu_seqlens_q=cu,
                                   seqlens_k=sk, max_seqlen_q=max_q)

    eager = call().clone()
    side = _side_stream(cuda, call)
    torch.cuda.synchronize()
    assert torch.equal(side, eager)
    g, gout = _capture(cuda, call)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(gout, eager)

    # shorter chunks over shorter pasts (the packed total stays within the captured buffer)
    past2, chunk2 = [40, 0, 2500], [200, 256, 1]
    cu.copy_(torch.tensor(np.concatenate([[0], np.cumsum(chunk2)]), dtype=torch.int32))
    sk.copy_(torch.tensor([p + c for p, c in zip(past2, chunk2)], dtype=torch.int32))
    sq.copy_(torch.randn(sum(chunk), hq, d, generator=gen, device=cuda).to(dtype))
    g.replay()
    torch.cuda.synchronize()
    replayed = gout.clone()
    eager2 = call()
    torch.cuda.synchronize()
    used = sum(chunk2)
    assert torch.equal(replayed[:used], eager2[:used])
    qn, kn, vn = (t.float().cpu().numpy() for t in (sq, kc, vc))
    qo = 0
    for b in range(B):
        tot = past2[b] + chunk2[b]
        pages = bt[b, :math.ceil(tot / 16)]
        kb = kn[pages].reshape(-1, hkv, d)[:tot]
        vb = vn[pages].reshape(-1, hkv, d)[:tot]
        ref = chunk_attention(qn[qo:qo + chunk2[b]], kb, vb)
        assert _err(replayed[qo:qo + chunk2[b]].float().cpu().numpy(), ref) < 2e-3
        qo += chunk2[b]
