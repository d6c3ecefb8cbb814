"""CPU tests of the selected-writeback host logic (no kernel runs): the
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
