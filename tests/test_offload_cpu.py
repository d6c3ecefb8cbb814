"""CPU tests of the offload manager's host logic: decode-slot bookkeeping
(reserve_decode_slot, core/offload.py:780-866; eviction loop :257-287), the
reference's registration, residency and per-layer decode-append calls
(:451-510, :307-360, :868-960), ensure / prefetch on resident or unknown
sequences, and the slot helpers.  The manager is built without its CUDA
transfer stream (only host state is touched here) over a CPU-device pool."""
import threading

import torch

from unifiedkv_b200.kv_types import BlockTableEntry, OffloadState
from unifiedkv_b200.offload import AsyncOffloadManager
from unifiedkv_b200.pool import PagedKVPool


def _manager(n_total=40, layers=3):
    pool = PagedKVPool(16, layers, 2, 64, torch.bfloat16, device="cpu", n_total=n_total)
    m = AsyncOffloadManager.__new__(AsyncOffloadManager)
    m.pool, m.num_layers, m.lock = pool, layers, threading.Lock()
    m.page_table, m._pending, m._stats, m._slot_of = {}, {}, {}, {}
    m._free_slots = list(range(8))
    return m


def _register(m, seq_id, n_pages, seq_len):
    ids = m.pool.allocate_blocks(n_pages)
    m.register_sequence(seq_id, ids, seq_len)
    return ids


def test_new_page_only_at_a_page_boundary():
    m = _manager()
    ids = _register(m, 1, 2, 32)
    free0 = m.pool.n_free
    r = m.reserve_decode_slot(1)
    assert r.ok and m.pool.n_free == free0 - 1
    new = m.page_table[(1, 0)].block_ids[-1]
    for l in range(3):  # the same new page id in every layer
        e = m.page_table[(1, l)]
        assert e.block_ids == ids + [new] and e.gpu_block_map == ids + [new] and e.materialized_blocks == 3
        assert e.state == OffloadState.ON_GPU
    m.commit_decode_token(1)
    assert all(m.page_table[(1, l)].seq_len == 33 for l in range(3))
    assert m.reserve_decode_slot(1).ok and m.pool.n_free == free0 - 1  # 33 % 16 != 0: no new page


def test_failure_reasons_follow_the_reference():
    m = _manager()
    r = m.reserve_decode_slot(9)
    assert (r.ok, r.retryable, r.reason) == (False, False, "missing_page_table_entry seq=9")
    _register(m, 2, 1, 10)
    m.page_table[(2, 1)].state = OffloadState.MIXED
    r = m.reserve_decode_slot(2)
    assert not r.ok and r.retryable and r.reason.startswith("direct_decode_not_on_gpu seq=2 state=")
    m.page_table[(2, 1)].state = OffloadState.ON_GPU
    m.page_table[(2, 2)].gpu_block_map[0] = -1
    r = m.reserve_decode_slot(2)
    assert (r.ok, r.retryable, r.reason) == (False, True, "direct_decode_resident_missing seq=2")
    m.page_table[(2, 2)].gpu_block_map[0] = m.page_table[(2, 2)].block_ids[0]
    m.page_table[(2, 0)].seq_len = 11
    r = m.reserve_decode_slot(2)
    assert (r.ok, r.retryable, r.reason) == (False, False, "direct_decode_inconsistent_seq_len seq=2")
    st = m.get_stats()
    assert st["decode_append_fail"] == 4 and st["decode_append_retryable"] == 2


def test_full_pool_evicts_or_reports():
    m = _manager(n_total=4)
    _register(m, 1, 4, 64)  # the pool is full and the last page is full
    r = m.reserve_decode_slot(1)  # no pressure policy supplied: nothing can be evicted
    assert (r.ok, r.retryable, r.reason) == (False, True, "direct_decode_expand_evict_failed")
    # a pressure policy that frees a victim's pages: eviction runs to max(high watermark, 1) free pages
    m2 = _manager(n_total=8)
    victim_pages = _register(m2, 7, 4, 64)
    _register(m2, 1, 4, 64)
    calls = []

    def evict_coldest_sequence(exclude_seq, protected_seqs=None):
        calls.append((exclude_seq, tuple(protected_seqs or ())))
        m2.pool.free_blocks_by_ids(victim_pages)
        return 7

    m2.evict_coldest_sequence = evict_coldest_sequence
    assert m2.pool.N_wm_high == 3
    r = m2.reserve_decode_slot(1)
    assert r.ok and calls == [(1, (1,))] and m2.pool.n_free == 3
    # a policy that frees nothing: the loop stops instead of spinning
    m3 = _manager(n_total=4)
    _register(m3, 1, 4, 64)
    m3.evict_coldest_sequence = lambda exclude_seq, protected_seqs=None: 5
    r = m3.reserve_decode_slot(1)
    assert r.reason == "direct_decode_expand_evict_failed" and m3.get_stats()["evict_fail"] == 1


def test_slot_helpers():
    m = _manager()
    m._free_slots = [5, 1, 2, 7, 3]
    assert m._alloc_slots(3) == [1, 2, 3] and m._free_slots == [5, 7]
    assert m._alloc_slots(3) is None and m._free_slots == [5, 7]
    assert AsyncOffloadManager._runs([1, 2, 3, 7, 9, 10]) == [(0, 1, 3), (3, 7, 1), (4, 9, 2)]
    e = BlockTableEntry(seq_id=1, layer_id=0, state=OffloadState.ON_GPU, block_ids=[4, 5], seq_len=20,
                        logical_seq_len=20, materialized_blocks=2, gpu_block_map=[4, -1],
                        cpu_k_blocks=[None, None], cpu_v_blocks=[None, None])
    AsyncOffloadManager._update_entry_state(e)
    assert e.state == OffloadState.MIXED
    e.gpu_block_map = [-1, -1]
    AsyncOffloadManager._update_entry_state(e)
    assert e.state == OffloadState.ON_CPU


def _torch_page_writes(pool):
    """Stand-in for the copy kernel behind write_kv_to_blocks: the reference's page
    loop (core/pool.py:127-142); the kernel path has its own GPU test."""
    def write_kv_to_blocks(layer_id, block_ids, K, V):
        for i, bid in enumerate(block_ids):
            s, e = 16 * i, min(16 * i + 16, K.shape[1])
            if e > s:
                pool.k_cache[layer_id, bid, :e - s] = K[:, s:e].transpose(0, 1)
                pool.v_cache[layer_id, bid, :e - s] = V[:, s:e].transpose(0, 1)
    pool.write_kv_to_blocks = write_kv_to_blocks


def test_register_residency_and_append_decode_token():
    m = _manager(n_total=12, layers=2)
    _torch_page_writes(m.pool)
    g = torch.Generator().manual_seed(1)
    K = [torch.randn(2, 31, 64, generator=g).to(torch.bfloat16) for _ in range(2)]
    V = [torch.randn(2, 31, 64, generator=g).to(torch.bfloat16) for _ in range(2)]
    ids = m.pool.allocate_blocks(2)
    m.register_all_layers(4, ids, 31, [K[0], None], [V[0], None], anchor_k_means=[torch.ones(64), None])
    assert (4, 0) in m.page_table and (4, 1) not in m.page_table  # a None layer is skipped
    assert torch.equal(m.page_table[(4, 0)].prefill_anchor_k_mean, torch.ones(64))
    got = m.register(4, 1, K[1], V[1])  # the reference's per-layer registration takes its own pages
    assert len(got) == 2 and m.pool.n_free == 8
    kb, _ = m.pool.read_kv_from_blocks(1, got, 31)
    assert torch.equal(kb, K[1])
    res = m.get_sequence_residency(4)
    assert res == dict(exists=1, on_gpu=1, resident_blocks=2, logical_blocks=2, materialized_blocks=2,
                       resident_ratio_x1000=1000, has_cpu_blocks=0, state_mixed=0, last_access=0,
                       residency_protected=0)
    assert m.get_sequence_residency(99)["exists"] == 0
    # decode tokens: position 31 fills the last page, 32 needs a new one (taken by layer 0)
    toks = [(torch.randn(2, 1, 64, generator=g).to(torch.bfloat16),
             torch.randn(2, 1, 64, generator=g).to(torch.bfloat16)) for _ in range(4)]
    for t in range(2):
        for layer in range(2):
            assert m.append_decode_token(4, layer, *toks[2 * t + layer]).ok
    e0, e1 = m.page_table[(4, 0)], m.page_table[(4, 1)]
    assert e0.seq_len == e1.seq_len == 33 and len(e0.block_ids) == 3 and len(e1.block_ids) == 3
    assert e0.block_ids[-1] == e1.block_ids[-1]  # one new page, shared by the layers
    assert torch.equal(m.pool.k_cache[1, e1.block_ids[-1], 0], toks[3][0][:, 0])
    assert torch.equal(m.pool.k_cache[0, e0.block_ids[1], 15], toks[0][0][:, 0])
    assert m.get_stats()["decode_append_success"] == 4
    # reasons of the reference
    r = m.append_decode_token(9, 0, *toks[0])
    assert (r.ok, r.retryable, r.reason) == (False, False, "missing_page_table_entry seq=9 layer=0")
    e0.gpu_block_map[0] = -1  # a page that is nowhere: neither resident nor in a host slot
    e0.state = OffloadState.MIXED
    r = m.append_decode_token(4, 0, *toks[0])
    assert (r.ok, r.retryable, r.reason) == (False, True, "prefetch_before_decode_append_failed seq=4")
    assert m.get_sequence_residency(4)["state_mixed"] == 1
    m2 = _manager(n_total=2, layers=1)
    m2.register_sequence(1, m2.pool.allocate_blocks(2), 32)
    r = m2.append_decode_token(1, 0, *toks[0])
    assert (r.ok, r.reason) == (False, "decode_expand_evict_failed")
    m3 = _manager(n_total=2, layers=1)
    m3.register_sequence(1, [], 0)
    r = m3.append_decode_token(1, 0, *toks[0])
    assert (r.ok, r.retryable, r.reason) == (False, True, "no_gpu_blocks_for_decode_append seq=1 layer=0")
    import pytest
    with pytest.raises(MemoryError, match="GPU blocks exhausted: seq=2 layer=0"):
        m3.register(2, 0, torch.zeros(2, 40, 64), torch.zeros(2, 40, 64))


def test_ensure_and_prefetch_on_unknown_or_resident_sequences():
    m = _manager()
    assert m.ensure_sequence_on_gpu(5) is False and m.get_stats()["ensure_fail"] == 1
    assert m.prefetch_sequence(5) is True  # nothing registered: a no-op success, as in the reference
    _register(m, 6, 2, 20)
    assert m.ensure_sequence_on_gpu(6) is True  # all pages resident: nothing to fetch
    assert m.prefetch_sequence(6) is True
