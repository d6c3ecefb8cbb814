"""CPU tests of the selected-writeback host logic (no kernel runs): the budget
rules against the reference's own table and the oracle, the
transaction's rollback (core/scheduler.py:805-878), the writeback allocation
with watermark eviction (core/scheduler.py:654-664) and its failure mode.
A CPU-device pool exercises the allocator; every case below fails or returns
before the first compaction launch."""
import pytest
import torch

from unifiedkv_b200.pool import PagedKVPool
from unifiedkv_b200.selection import SelectionEngine


def _engine(n_total=100, layers=2):
    pool = PagedKVPool(16, layers, 2, 64, torch.bfloat16, device="cpu", n_total=n_total)
    return SelectionEngine(pool, num_q_heads=8, sink_len=16, obs_len=16, retain_ratio=0.25)


def _raw(layers, L=1000):
    return {l: (torch.zeros(2, L, 64), torch.zeros(2, L, 64)) for l in range(layers)}


def test_forced_oom_rolls_back(monkeypatch):
    eng = _engine()
    monkeypatch.setenv("KV_MIDDLEWARE_FORCE_GPU_WRITEBACK_OOM", "1")
    with pytest.raises(torch.cuda.OutOfMemoryError):
        eng._selected_writeback_transaction(3, _raw(2), {0: [0], 1: [0]}, 48, 1000, "ratio")
    assert eng.pool.n_free == 100  # the three pages taken for the writeback went back
    assert eng.writeback_transaction_rollbacks == 1 and eng.page_table == {}


def test_missing_layer_rolls_back():
    eng = _engine()
    with pytest.raises(RuntimeError, match="selected_writeback_missing_raw seq=5 layer=0"):
        eng._selected_writeback_transaction(5, {}, {}, 48, 1000, "ratio")
    assert eng.pool.n_free == 100 and eng.writeback_transaction_rollbacks == 1 and eng.page_table == {}


def test_allocation_failure_takes_nothing():
    eng = _engine(n_total=10)
    with pytest.raises(MemoryError, match="Cannot allocate 11 blocks for seq=7"):
        eng._allocate_writeback_blocks(7, 11)
    assert eng.pool.n_free == 10


def test_watermark_eviction_before_allocation():
    """Below the low watermark, victims are evicted until max(n_req, high watermark)
    pages are free; then the request is served from the FIFO free list."""
    eng = _engine(n_total=100)
    pool = eng.pool
    victims = [pool.allocate_blocks(10) for _ in range(9)]  # 90 taken, 10 free < N_wm_low = 15
    assert pool.n_free == 10 and (pool.N_wm_low, pool.N_wm_high) == (15, 40)
    calls = []

    def evict(seq_id, target):
        calls.append((seq_id, target))
        pool.free_blocks_by_ids(victims.pop(0))

    eng._evict_one_for_prefill_allocation = evict
    ids = eng._allocate_writeback_blocks(4, 3)
    assert calls == [(4, 40)] * 3  # 10 -> 20 -> 30 -> 40 free
    assert len(ids) == 3 and pool.n_free == 37
    # above the low watermark: evict only while fewer than n_req pages are free
    calls.clear()
    ids2 = eng._allocate_writeback_blocks(4, 20)
    assert calls == [] and len(ids2) == 20 and pool.n_free == 17


def test_budget_rule_matches_the_reference_table():
    """SelectedWritebackOps._selection_budget_blocks against the table generated
    from the reference's own KVScheduler._selection_budget_blocks
    (core/scheduler.py:547-564; tests/golden/budget.json)."""
    import json
    from pathlib import Path
    rows = json.loads((Path(__file__).parent / "golden" / "budget.json").read_text())
    pool = PagedKVPool(16, 1, 2, 64, torch.bfloat16, device="cpu", n_total=4)
    for r in rows:
        eng = SelectionEngine(pool, num_q_heads=8, sink_len=r["sink"], obs_len=r["obs"], retain_ratio=r["ratio"],
                              retain_budget_tokens=r["budget"])
        assert eng._selection_budget_blocks(r["L"]) == (r["k"], r["eff"], r["mode"]), r


def test_compress_k_blocks_matches_the_oracle():
    """BlockAlignedSnapKV's k rule (core/compress.py:133-139) on a grid, against the
    oracle pinned to the reference's compress fixtures."""
    from oracle import compress as oc
    from unifiedkv_b200.compress import BlockAlignedSnapKV
    for N in (0, 1, 5, 16, 511, 2044, 2045):
        for sink, obs in ((64, 64), (16, 16), (0, 0), (7, 13)):
            for budget in (0, 100, 2048, 8192):
                for ratio in (0.01, 0.2, 0.25, 1.0):
                    c = BlockAlignedSnapKV(16, sink, obs, retain_ratio=ratio, retain_budget_tokens=budget)
                    k, mode = c._k_blocks(N)
                    assert k == oc.compress_k_blocks(N, sink, obs, budget, ratio), (N, sink, obs, budget, ratio)
                    assert mode == c.compression_mode == ("fixed_budget" if budget > 0 else "ratio")


def test_block_indexed_writeback_declines_like_the_reference():
    """_write_block_indexed_layer_to_pool (core/scheduler.py:702-733) returns False,
    writing nothing, when the aligned fast path does not apply: no sources, a
    source/page count mismatch, a length that is not whole pages, a source block
    out of range."""
    eng = _engine()
    K = torch.zeros(2, 64, 64)
    before = eng.pool.k_cache.clone()
    assert not eng._write_block_indexed_layer_to_pool(0, [1, 2], K, K, [])
    assert not eng._write_block_indexed_layer_to_pool(0, [1, 2], K, K, [0])
    assert not eng._write_block_indexed_layer_to_pool(0, [1], K[:, :60], K[:, :60], [0])
    assert not eng._write_block_indexed_layer_to_pool(0, [1], K, K, [4])
    assert not eng._write_block_indexed_layer_to_pool(0, [1, 2], K, K, [-1, 3])
    assert torch.equal(eng.pool.k_cache, before)
