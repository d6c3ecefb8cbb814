"""CPU tests: compression/selection/writeback oracle against golden vectors
produced by the reference's own code (tests/golden/make_golden.py)."""
import json
from pathlib import Path

import numpy as np
import pytest

from oracle import compress as oc
from tests.golden.inputs import checksum, compress_case

GOLDEN = Path(__file__).parent / "golden"
SPECS = {
    "regression_l2795": dict(seed=7, h_kv=8, L=2795, d=32, n_rep=4, window=16),
    "ratio_l4100": dict(seed=11, h_kv=8, L=4100, d=64, n_rep=4, window=64),
    "hot_l8192": dict(seed=5, h_kv=8, L=8192, d=128, n_rep=4, window=64, hot_blocks=16, sink=64),
    "skip_le_budget": dict(seed=3, h_kv=2, L=600, d=32, n_rep=2, window=16),
}


@pytest.mark.parametrize("name", sorted(SPECS))
def test_compress_matches_reference(name):
    g = np.load(GOLDEN / f"compress_{name}.npz")
    K, V, Q, _ = compress_case(**SPECS[name])
    assert str(g["inputs_sha"]) == checksum(K, V, Q)
    params = json.loads(str(g["params"]))
    budget = params.get("retain_budget_tokens", 0)
    ratio = params.get("retain_ratio", 0.2)
    res = oc.compress(K.astype(np.float64), V.astype(np.float64), Q.astype(np.float64), params["sink_len"],
                      params["obs_len"], budget, ratio)
    Kf, Vf, sel = res
    ref_idx = g["retained_block_idx"]
    if sel is None:
        assert len(ref_idx) == 0 and Kf.shape[1] == int(g["k_final_len"])
        return
    assert Kf.shape[1] == int(g["k_final_len"])
    if not np.array_equal(sel, ref_idx):
        # torch.topk leaves the order of exactly tied scores unspecified (max-pool
        # creates exact copies); the oracle keeps the lowest index.  Only such
        # exact ties at the k-th score may differ.
        scores = oc.block_scores(K, Q, params["sink_len"], params["obs_len"])
        diff = set(sel.tolist()) ^ set(ref_idx.tolist())
        kth = np.sort(scores)[::-1][len(sel) - 1]
        assert all(abs(scores[i] - kth) <= 1e-12 * kth for i in diff), diff
        assert oc.selection_is_consistent(ref_idx, scores, len(sel), rel_tol=1e-12)
        return
    # K_final identical to the reference's output bytes (gather of fp32 rows)
    assert checksum(Kf.astype(np.float32)) == str(g["k_final_sha"])
    assert checksum(Vf.astype(np.float32)) == str(g["v_final_sha"])
    dbg = json.loads(str(g["debug"]))
    N = int(np.ceil((K.shape[1] - params["sink_len"] - params["obs_len"]) / 16))
    assert dbg["mid_block_count"] == N and dbg["retained_block_count"] == len(sel)


def test_regression_debug_fields():
    """benchmarks/test_block_alignment_regression.py:37-47 invariants."""
    dbg = json.loads(str(np.load(GOLDEN / "compress_regression_l2795.npz")["debug"]))
    mid = 2795 - 16 - 16
    assert dbg["mid_tokens_before_align"] == mid
    assert dbg["mid_tokens_aligned"] == (mid + 15) // 16 * 16
    assert dbg["effective_retained_tokens"] == 2048


@pytest.mark.parametrize("name,sink,obs", [("l2795_d32", 16, 16), ("l4100_d64", 64, 64)])
def test_scores_match_scheduler(name, sink, obs):
    g = np.load(GOLDEN / f"score_{name}.npz")
    spec = json.loads(str(g["spec"]))
    K, V, Q, _ = compress_case(seed=spec["seed"], h_kv=spec["h_kv"], L=spec["L"], d=spec["d"], n_rep=spec["n_rep"],
                               window=spec["window"])
    s = oc.block_scores(K, Q, sink, obs, smooth="if3")
    assert np.allclose(s, g["score"], rtol=2e-5, atol=1e-7)


def test_budget_table_matches_scheduler():
    rows = json.loads((GOLDEN / "budget.json").read_text())
    for r in rows:
        k, eff, mode = oc.selection_budget_blocks(r["L"], r["sink"], r["obs"], r["budget"], r["ratio"])
        assert (k, eff, mode) == (r["k"], r["eff"], r["mode"]), r


@pytest.mark.parametrize("name", ["aligned", "unaligned", "odd_sink"])
def test_writeback_matches_scheduler(name):
    g = np.load(GOLDEN / f"writeback_{name}.npz")
    K, V = g["K"], g["V"]
    src = oc.writeback_source_tokens(K.shape[1], int(g["sink"]), int(g["obs"]), g["selected"])
    assert len(src) == int(g["eff"])
    init_k = np.full_like(g["k_pool"], -7.0)
    init_v = np.full_like(g["v_pool"], -9.0)
    kp, vp = oc.writeback_pool(init_k, init_v, K, V, g["dst"], src)
    assert np.array_equal(kp, g["k_pool"]) and np.array_equal(vp, g["v_pool"])


def test_topk_ties_lowest_index():
    s = np.array([1.0, 3.0, 3.0, 2.0, 3.0, 0.5])
    assert list(oc.topk_lowest_index(s, 2)) == [1, 2]
    assert list(oc.topk_lowest_index(s, 4)) == [1, 2, 3, 4]


def test_per_kv_head_oracle_reduces_to_shared():
    """Per-KV-head mode (no reference counterpart): with one KV head it is the
    shared mode; with several, the shared (unsmoothed) block score bounds every
    head's, and each head's selection is the top-k of its own row."""
    from tests.golden.inputs import compress_case
    K, V, Q, _ = compress_case(seed=4, h_kv=1, L=600, d=32, n_rep=4, window=8)
    np.testing.assert_array_equal(oc.block_scores(K, Q, 16, 16, per_kv_head=True)[0], oc.block_scores(K, Q, 16, 16))
    Kf, Vf, sel = oc.compress_per_kv_head(K, V, Q, 16, 16, ratio=0.25)
    Kg, Vg, selg = oc.compress(K, V, Q, 16, 16, ratio=0.25)
    np.testing.assert_array_equal(sel[0], selg)
    np.testing.assert_array_equal(Kf, Kg)
    K, V, Q, _ = compress_case(seed=5, h_kv=3, L=900, d=32, n_rep=2, window=8)
    sh = oc.block_scores(K, Q, 16, 16, smooth="never")
    ph = oc.block_scores(K, Q, 16, 16, smooth="never", per_kv_head=True)
    assert ph.shape == (3, sh.shape[0]) and np.all(sh >= ph.max(axis=0) - 1e-15)
    Kf, Vf, sel = oc.compress_per_kv_head(K, V, Q, 16, 16, ratio=0.25)
    scores = oc.block_scores(K, Q, 16, 16, per_kv_head=True)
    for h in range(3):
        np.testing.assert_array_equal(sel[h], oc.topk_lowest_index(scores[h], sel.shape[1]))
        src = oc.writeback_source_tokens(900, 16, 16, sel[h])
        np.testing.assert_array_equal(Kf[h], np.where(src[:, None] >= 0, K[h, np.maximum(src, 0)], 0))


@pytest.mark.parametrize("name", ["ratio_l4100", "hot_l8192"])
def test_per_kv_head_matches_reference_per_head(name):
    """Per-KV-head selection pinned to the reference's own code: for KV head h it keeps
    what BlockAlignedSnapKV.compress keeps when given head h alone with its group's
    query heads (golden: tests/golden/compress_perhead_*.npz)."""
    g = np.load(GOLDEN / f"compress_perhead_{name}.npz")
    K, V, Q, _ = compress_case(**SPECS[name])
    assert str(g["inputs_sha"]) == checksum(K, V, Q)
    params = json.loads(str(g["params"]))
    budget = params.get("retain_budget_tokens", 0)
    ratio = params.get("retain_ratio", 0.2)
    sink, obs = params["sink_len"], params["obs_len"]
    Kf, Vf, sel = oc.compress_per_kv_head(K.astype(np.float64), V.astype(np.float64), Q.astype(np.float64), sink,
                                          obs, budget, ratio)
    ref = g["retained_block_idx"]
    assert sel.shape == ref.shape
    scores = oc.block_scores(K, Q, sink, obs, per_kv_head=True)
    for h in range(K.shape[0]):
        assert Kf.shape[1] == int(g["k_final_len"][h])
        if np.array_equal(sel[h], ref[h]):
            assert checksum(Kf[h:h + 1].astype(np.float32)) == str(g["k_final_sha"][h])
            assert checksum(Vf[h:h + 1].astype(np.float32)) == str(g["v_final_sha"][h])
            continue
        # only exact ties at the k-th score may differ (torch.topk's order is unspecified)
        diff = set(sel[h].tolist()) ^ set(ref[h].tolist())
        kth = np.sort(scores[h])[::-1][sel.shape[1] - 1]
        assert all(abs(scores[h][i] - kth) <= 1e-12 * kth for i in diff), (h, diff)
