"""GPU parity of block scoring, top-k selection and compacting writeback.

Bars: top-k and writeback are bit-exact against the oracle on identical
inputs; block scores match the fp64 oracle of the same (rounded) inputs to a
relative 1e-4, and the selected set equals the oracle's except where fp64
scores lie within 1e-4 (relative) of the k-th score (near-ties that a different
float summation order may flip; exact ties always go to the lowest index).
"""
import json
import math
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import compress as oc
from tests.golden.inputs import compress_case

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).parent / "golden"


def _t(x, cuda, dtype):
    return torch.from_numpy(np.ascontiguousarray(x, np.float32)).to(cuda, dtype)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("spec", [
    dict(seed=7, h_kv=8, L=2795, d=32, n_rep=4, window=16, sink=16, obs=16),
    dict(seed=11, h_kv=8, L=4100, d=64, n_rep=4, window=64, sink=64, obs=64),
    dict(seed=12, h_kv=2, L=1000, d=128, n_rep=8, window=20, sink=7, obs=13),
    dict(seed=13, h_kv=4, L=70, d=256, n_rep=1, window=3, sink=16, obs=16),
])
def test_block_scores(cuda, dtype, spec):
    from unifiedkv_b200.compress import SMOOTH_ALWAYS, block_scores
    K, V, Q, _ = compress_case(seed=spec["seed"], h_kv=spec["h_kv"], L=spec["L"], d=spec["d"], n_rep=spec["n_rep"],
                               window=spec["window"])
    tk, tq = _t(K, cuda, dtype), _t(Q, cuda, dtype)
    s = block_scores(tk, tq, spec["sink"], spec["obs"], smooth=SMOOTH_ALWAYS)
    s2 = block_scores(tk, tq, spec["sink"], spec["obs"], smooth=SMOOTH_ALWAYS)
    torch.cuda.synchronize()
    assert torch.equal(s, s2), "scores must be bit-reproducible"
    ref = oc.block_scores(tk.float().cpu().numpy(), tq.float().cpu().numpy(), spec["sink"], spec["obs"])
    got = s.cpu().numpy()
    assert got.shape == ref.shape
    assert np.allclose(got, ref, rtol=1e-4, atol=1e-7), np.max(np.abs(got - ref) / ref)


@pytest.mark.parametrize("n,k", [(1, 1), (5, 2), (173, 40), (2044, 511), (3000, 1), (16384, 4096), (49152, 30000), (100, 0)])
def test_topk_bit_exact_with_ties(cuda, n, k):
    from unifiedkv_b200.compress import topk_blocks
    rng = np.random.default_rng(n + k)
    s = rng.standard_normal(n).astype(np.float32)
    s[rng.integers(0, n, size=n // 3)] = 0.5  # many exact ties
    if n > 10:
        s[3] = np.inf
        s[4] = -np.inf
        s[5] = -0.0
        s[6] = 0.0
    got = topk_blocks(torch.from_numpy(s).to(cuda), k).cpu().numpy()
    assert np.array_equal(got, oc.topk_lowest_index(s, k))


def test_topk_all_equal(cuda):
    from unifiedkv_b200.compress import topk_blocks
    s = torch.ones(999, device=cuda)
    assert topk_blocks(s, 10).cpu().tolist() == list(range(10))


@pytest.mark.parametrize("name", ["aligned", "unaligned", "odd_sink"])
def test_writeback_bit_exact_vs_reference_fixture(cuda, name):
    from unifiedkv_b200.pool import write_pages
    g = np.load(GOLDEN / f"writeback_{name}.npz")
    K, V = torch.from_numpy(g["K"]).to(cuda), torch.from_numpy(g["V"]).to(cuda)
    kp = torch.full(g["k_pool"].shape, -7.0, device=cuda)
    vp = torch.full(g["v_pool"].shape, -9.0, device=cuda)
    sel = torch.from_numpy(g["selected"].astype(np.int32)).to(cuda)
    write_pages(kp, vp, K, V, g["dst"].tolist(), sel, int(sel.numel()), int(g["sink"]), int(g["obs"]))
    torch.cuda.synchronize()
    assert np.array_equal(kp.cpu().numpy(), g["k_pool"]) and np.array_equal(vp.cpu().numpy(), g["v_pool"])


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_compress_end_to_end(cuda, dtype):
    from unifiedkv_b200.compress import BlockAlignedSnapKV
    K, V, Q, hot = compress_case(seed=5, h_kv=8, L=8192, d=128, n_rep=4, window=64, hot_blocks=16, sink=64)
    tk, tv, tq = _t(K, cuda, dtype), _t(V, cuda, dtype), _t(Q, cuda, dtype)
    c = BlockAlignedSnapKV(16, 64, 64, retain_ratio=0.25)
    Kf, Vf = c.compress(tk[None], tv[None], tq[None], n_rep=4)
    sel = np.asarray(c.last_debug["retained_block_idx"][0])
    Kr, Vr, Qr = (t.float().cpu().numpy() for t in (tk, tv, tq))
    scores = oc.block_scores(Kr, Qr, 64, 64)
    k = c.last_debug["retained_block_count"]
    assert k == oc.compress_k_blocks(len(scores), 64, 64, 0, 0.25)
    assert oc.selection_is_consistent(sel, scores, k, rel_tol=1e-4)
    hot_mid = hot - 4
    hot_mid = hot_mid[(hot_mid >= 0) & (hot_mid < len(scores))]
    assert set(hot_mid.tolist()) <= set(sel.tolist()), "hot blocks must be retained"
    src = oc.writeback_source_tokens(8192, 64, 64, sel)
    ref_k = np.where(src[None, :, None] >= 0, Kr[:, np.maximum(src, 0)], 0)
    ref_v = np.where(src[None, :, None] >= 0, Vr[:, np.maximum(src, 0)], 0)
    assert np.array_equal(Kf[0].float().cpu().numpy(), ref_k)
    assert np.array_equal(Vf[0].float().cpu().numpy(), ref_v)
    assert c.last_debug["mid_tokens_aligned"] == len(scores) * 16


def test_compress_skip_and_regression_shape(cuda):
    """benchmarks/test_block_alignment_regression.py contract on the GPU path."""
    from unifiedkv_b200.compress import BlockAlignedSnapKV
    K, V, Q, _ = compress_case(seed=7, h_kv=8, L=2795, d=32, n_rep=4, window=16)
    c = BlockAlignedSnapKV(16, 16, 16, retain_budget_tokens=2048)
    Kf, Vf = c.compress(_t(K, cuda, torch.float16)[None], _t(V, cuda, torch.float16)[None],
                        _t(Q, cuda, torch.float16)[None], n_rep=4)
    mid = 2795 - 32
    assert c.last_debug["mid_tokens_before_align"] == mid
    assert c.last_debug["mid_tokens_aligned"] == (mid + 15) // 16 * 16
    assert max(c.last_debug["retained_block_idx"][0]) < (mid + 15) // 16
    assert Kf.shape == Vf.shape and Kf.shape[2] == 2048
    c2 = BlockAlignedSnapKV(16, 16, 16, retain_budget_tokens=4096)
    Kf2, _ = c2.compress(_t(K, cuda, torch.float16)[None], _t(V, cuda, torch.float16)[None],
                         _t(Q, cuda, torch.float16)[None], n_rep=4)
    assert Kf2.shape[2] == 2795 and c2.last_debug["compression_skipped"] == "input_le_budget"


def test_config4_full_size_selection(cuda):
    """32768 tokens, 8 KV heads, d=128, 64-query window over 32 q-heads, 32 hot
    blocks at +2 sigma; keep 25% of mid blocks plus first 4 and last 8 blocks."""
    from unifiedkv_b200.compress import SMOOTH_ALWAYS, block_scores, topk_blocks
    K, V, Q, hot = compress_case(seed=4, h_kv=8, L=32768, d=128, n_rep=4, window=64, hot_blocks=32, sink=64)
    tk, tq = _t(K, cuda, torch.bfloat16), _t(Q, cuda, torch.bfloat16)
    s = block_scores(tk, tq, 64, 128, smooth=SMOOTH_ALWAYS)
    N = s.numel()
    k = int(math.floor(0.25 * N))
    sel = topk_blocks(s, k).cpu().numpy()
    ref = oc.block_scores(tk.float().cpu().numpy(), tq.float().cpu().numpy(), 64, 128, dtype=np.float64)
    assert np.allclose(s.cpu().numpy(), ref, rtol=1e-4)
    assert oc.selection_is_consistent(sel, ref, k, rel_tol=1e-4)
    hot_mid = hot - 4
    hot_mid = hot_mid[(hot_mid >= 0) & (hot_mid < N)]
    assert set(hot_mid.tolist()) <= set(sel.tolist())


def test_selection_engine_transaction(cuda, monkeypatch):
    from unifiedkv_b200.pool import PagedKVPool
    from unifiedkv_b200.selection import SelectionEngine
    layers, h_kv, d, L = 3, 2, 64, 1000
    pool = PagedKVPool(16, layers, h_kv, d, torch.bfloat16, device=cuda, n_total=200)
    eng = SelectionEngine(pool, num_q_heads=8, sink_len=16, obs_len=16, retain_ratio=0.25)
    rng = np.random.default_rng(0)
    raw = {}
    for l in range(layers):
        K = _t(rng.standard_normal((h_kv, L, d)), cuda, torch.bfloat16)
        V = _t(rng.standard_normal((h_kv, L, d)), cuda, torch.bfloat16)
        raw[l] = (K, V)
        eng.q_cache[l][7] = _t(rng.standard_normal((8, L, d)), cuda, torch.bfloat16)
    ids, selected, eff = eng.select_and_writeback(7, raw)
    k, eff_ref, mode = oc.selection_budget_blocks(L, 16, 16, 0, 0.25)
    assert eff == eff_ref and len(ids) == math.ceil(eff / 16)
    for l in range(layers):
        K, V = (t.float().cpu().numpy() for t in raw[l])
        Qo = eng.q_cache[l][7][:, -16:].float().cpu().numpy()
        sc = oc.block_scores(K, Qo, 16, 16, smooth="if3")
        assert oc.selection_is_consistent(np.array(selected[l]), sc, k, rel_tol=1e-4)
        src = oc.writeback_source_tokens(L, 16, 16, selected[l])
        kp = pool.k_cache[l].float().cpu().numpy()
        for p, t in enumerate(src):
            want = K[:, t] if t >= 0 else np.zeros_like(K[:, 0])
            assert np.array_equal(kp[ids[p // 16], p % 16], want)
    assert eng.page_table[(7, 2)].seq_len == eff and eng.snapkv.last_debug["retained_block_count"] == k
    # forced OOM rolls the allocation back (core/scheduler.py:819-820, 872-878)
    free_before = pool.n_free
    monkeypatch.setenv("KV_MIDDLEWARE_FORCE_GPU_WRITEBACK_OOM", "1")
    with pytest.raises(torch.cuda.OutOfMemoryError):
        eng._selected_writeback_transaction(8, raw, selected, eff, L, "ratio")
    assert pool.n_free == free_before and eng.writeback_transaction_rollbacks == 1


def test_block_scores_large_logits(cuda):
    """Window queries 40x larger than usual: per-row maxima jump by far more than 2^8
    between K tiles, exercising the statistics pass's rescale and its recompute for
    jumps above 2^120; scores still match the fp64 oracle."""
    from unifiedkv_b200.compress import SMOOTH_ALWAYS, block_scores
    K, V, Q, _ = compress_case(seed=71, h_kv=8, L=6000, d=128, n_rep=4, window=64)
    ramp = np.linspace(0.1, 4.0, 6000, dtype=np.float32)[None, :, None]
    tk = _t(K * ramp, cuda, torch.bfloat16)
    tq = _t(Q * 40.0, cuda, torch.bfloat16)
    s = block_scores(tk, tq, 64, 64, smooth=SMOOTH_ALWAYS)
    torch.cuda.synchronize()
    ref = oc.block_scores(tk.float().cpu().numpy(), tq.float().cpu().numpy(), 64, 64)
    got = s.cpu().numpy()
    assert np.isfinite(got).all()
    # most blocks carry (close to) zero mass here: compare relative to the largest score
    assert np.max(np.abs(got - ref)) < 1e-4 * np.max(ref) + 1e-7, np.max(np.abs(got - ref))
