"""GPU parity of the per-KV-head selection mode (scores, batched top-k,
per-head compaction, BlockAlignedSnapKV(per_kv_head=True), SelectionEngine).

The reference shares one block selection across KV heads; this mode keeps the
top-k blocks of each KV head.  Bars as for the shared mode: per-head scores
match the fp64 oracle of the same rounded inputs to a relative 1e-4, top-k and
compaction are bit-exact, and a selected set may differ from the oracle's only
among fp64 scores within 1e-4 (relative) of that head's k-th score.
"""
import math

import numpy as np
import pytest
import torch

from oracle import compress as oc
from tests.golden.inputs import compress_case

pytestmark = pytest.mark.gpu


def _t(x, cuda, dtype):
    return torch.from_numpy(np.ascontiguousarray(x, np.float32)).to(cuda, dtype)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("spec", [
    dict(seed=21, h_kv=8, L=4100, d=128, n_rep=4, window=64, sink=64, obs=64),  # tcgen05 passes
    dict(seed=22, h_kv=4, L=1500, d=64, n_rep=2, window=32, sink=16, obs=16),   # mma.sync passes
    dict(seed=23, h_kv=2, L=333, d=128, n_rep=8, window=20, sink=7, obs=13),
])
def test_per_kv_head_scores(cuda, dtype, spec):
    from unifiedkv_b200.compress import SMOOTH_ALWAYS, SMOOTH_NONE, block_scores
    K, V, Q, _ = compress_case(seed=spec["seed"], h_kv=spec["h_kv"], L=spec["L"], d=spec["d"], n_rep=spec["n_rep"],
                               window=spec["window"])
    tk, tq = _t(K, cuda, dtype), _t(Q, cuda, dtype)
    s = block_scores(tk, tq, spec["sink"], spec["obs"], smooth=SMOOTH_ALWAYS, per_kv_head=True)
    s2 = block_scores(tk, tq, spec["sink"], spec["obs"], smooth=SMOOTH_ALWAYS, per_kv_head=True)
    torch.cuda.synchronize()
    assert torch.equal(s, s2), "scores must be bit-reproducible"
    Kr, Qr = tk.float().cpu().numpy(), tq.float().cpu().numpy()
    ref = oc.block_scores(Kr, Qr, spec["sink"], spec["obs"], per_kv_head=True)
    got = s.cpu().numpy()
    assert got.shape == ref.shape == (spec["h_kv"], math.ceil((spec["L"] - spec["sink"] - spec["obs"]) / 16))
    assert np.allclose(got, ref, rtol=1e-4, atol=1e-7), np.max(np.abs(got - ref) / ref)
    # the shared score sums the per-token max over KV groups, so it bounds every group's block sum
    sh = block_scores(tk, tq, spec["sink"], spec["obs"], smooth=SMOOTH_NONE).cpu().numpy()
    ph = block_scores(tk, tq, spec["sink"], spec["obs"], smooth=SMOOTH_NONE, per_kv_head=True).cpu().numpy()
    assert np.all(sh >= ph.max(axis=0) * (1 - 1e-5))


def test_topk_batched_bit_exact(cuda):
    from unifiedkv_b200.compress import topk_blocks
    rng = np.random.default_rng(3)
    s = rng.standard_normal((6, 777)).astype(np.float32)
    s[:, rng.integers(0, 777, size=200)] = 0.25  # exact ties in every row
    s[2] = 1.0  # an all-equal row
    got = topk_blocks(torch.from_numpy(s).to(cuda), 100).cpu().numpy()
    assert got.shape == (6, 100)
    for r in range(6):
        assert np.array_equal(got[r], oc.topk_lowest_index(s[r], 100))


@pytest.mark.parametrize("sink,obs,L", [(16, 16, 700), (7, 13, 555), (0, 0, 320)])
def test_per_kv_head_compaction_bit_exact(cuda, sink, obs, L):
    from unifiedkv_b200.pool import write_pages
    rng = np.random.default_rng(L)
    h_kv, d, n_pool = 4, 64, 120
    N = math.ceil((L - sink - obs) / 16)
    k = N // 3
    K = rng.standard_normal((h_kv, L, d)).astype(np.float32)
    V = rng.standard_normal((h_kv, L, d)).astype(np.float32)
    sel = np.stack([np.sort(rng.choice(N, k, replace=False)) for _ in range(h_kv)]).astype(np.int32)
    eff = sink + 16 * k + obs
    dst = rng.permutation(n_pool)[:math.ceil(eff / 16)].astype(np.int32)
    kp = torch.full((n_pool, 16, h_kv, d), -7.0, device=cuda)
    vp = torch.full((n_pool, 16, h_kv, d), -9.0, device=cuda)
    write_pages(kp, vp, torch.from_numpy(K).to(cuda), torch.from_numpy(V).to(cuda), dst.tolist(),
                torch.from_numpy(sel).to(cuda), k, sink, obs)
    torch.cuda.synchronize()
    src = np.stack([oc.writeback_source_tokens(L, sink, obs, sel[h]) for h in range(h_kv)])
    rk, rv = oc.writeback_pool(np.full((n_pool, 16, h_kv, d), -7.0, np.float32),
                               np.full((n_pool, 16, h_kv, d), -9.0, np.float32), K, V, dst, src)
    assert np.array_equal(kp.cpu().numpy(), rk) and np.array_equal(vp.cpu().numpy(), rv)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_compress_per_kv_head_end_to_end(cuda, dtype):
    from unifiedkv_b200.compress import BlockAlignedSnapKV
    K, V, Q, hot = compress_case(seed=9, h_kv=8, L=8192, d=128, n_rep=4, window=64, hot_blocks=16, sink=64)
    tk, tv, tq = _t(K, cuda, dtype), _t(V, cuda, dtype), _t(Q, cuda, dtype)
    c = BlockAlignedSnapKV(16, 64, 64, retain_ratio=0.25, per_kv_head=True)
    Kf, Vf = c.compress(tk[None], tv[None], tq[None], n_rep=4)
    sel = np.asarray(c.last_debug["retained_block_idx"][0])
    assert c.last_debug["selection_scope"] == "per_kv_head"
    Kr, Vr, Qr = (t.float().cpu().numpy() for t in (tk, tv, tq))
    scores = oc.block_scores(Kr, Qr, 64, 64, per_kv_head=True)
    k = c.last_debug["retained_block_count"]
    assert sel.shape == (8, k) and k == oc.compress_k_blocks(scores.shape[1], 64, 64, 0, 0.25)
    hot_mid = hot - 4
    hot_mid = hot_mid[(hot_mid >= 0) & (hot_mid < scores.shape[1])]
    for h in range(8):
        assert oc.selection_is_consistent(sel[h], scores[h], k, rel_tol=1e-4)
        assert set(hot_mid.tolist()) <= set(sel[h].tolist()), "hot blocks (hot for every head) must be retained"
        src = oc.writeback_source_tokens(8192, 64, 64, sel[h])
        assert np.array_equal(Kf[0, h].float().cpu().numpy(), np.where(src[:, None] >= 0, Kr[h, np.maximum(src, 0)], 0))
        assert np.array_equal(Vf[0, h].float().cpu().numpy(), np.where(src[:, None] >= 0, Vr[h, np.maximum(src, 0)], 0))
    # heads do pick different blocks in this mode
    assert any(not np.array_equal(sel[0], sel[h]) for h in range(1, 8))


def test_selection_engine_per_kv_head(cuda):
    from unifiedkv_b200.pool import PagedKVPool
    from unifiedkv_b200.selection import SelectionEngine
    layers, h_kv, d, L = 2, 2, 64, 1000
    pool = PagedKVPool(16, layers, h_kv, d, torch.bfloat16, device=cuda, n_total=200)
    eng = SelectionEngine(pool, num_q_heads=8, sink_len=16, obs_len=16, retain_ratio=0.25, per_kv_head=True)
    rng = np.random.default_rng(1)
    raw = {}
    for l in range(layers):
        raw[l] = (_t(rng.standard_normal((h_kv, L, d)), cuda, torch.bfloat16),
                  _t(rng.standard_normal((h_kv, L, d)), cuda, torch.bfloat16))
        eng.q_cache[l][3] = _t(rng.standard_normal((8, L, d)), cuda, torch.bfloat16)
    ids, selected, eff = eng.select_and_writeback(3, raw)
    k, eff_ref, _ = oc.selection_budget_blocks(L, 16, 16, 0, 0.25)
    assert eff == eff_ref and eng.snapkv.last_debug["selection_scope"] == "per_kv_head"
    for l in range(layers):
        K = raw[l][0].float().cpu().numpy()
        Qo = eng.q_cache[l][3][:, -16:].float().cpu().numpy()
        sc = oc.block_scores(K, Qo, 16, 16, smooth="if3", per_kv_head=True)
        kp = pool.k_cache[l].float().cpu().numpy()
        for h in range(h_kv):
            assert len(selected[l][h]) == k
            assert oc.selection_is_consistent(np.array(selected[l][h]), sc[h], k, rel_tol=1e-4)
            src = oc.writeback_source_tokens(L, 16, 16, selected[l][h])
            for p, t in enumerate(src):
                want = K[h, t] if t >= 0 else np.zeros_like(K[h, 0])
                assert np.array_equal(kp[ids[p // 16], p % 16, h], want)
