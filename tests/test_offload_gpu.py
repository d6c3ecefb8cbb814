"""Offload / prefetch of pool pages through pinned host slots (core/offload.py
mechanism, batched): round trips are bit-exact, freed pages return to the
pool, and Page16 decode over the prefetched pages equals decode before the
offload (the compute stream waits on the prefetch event, no host sync)."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _setup(cuda, layers=3, n_total=300, L=1000):
    from unifiedkv_b200.offload import AsyncOffloadManager
    from unifiedkv_b200.pool import PagedKVPool
    pool = PagedKVPool(16, layers, 8, 128, torch.bfloat16, device=cuda, n_total=n_total)
    g = torch.Generator(device=cuda).manual_seed(0)
    pool.k_cache.normal_(0, 0.5, generator=g)
    pool.v_cache.normal_(0, 0.5, generator=g)
    mgr = AsyncOffloadManager(pool, layers, host_slots=128, staging_pages=7)  # small staging: chunked path
    ids = pool.allocate_blocks((L + 15) // 16)
    mgr.register_sequence(1, ids, L)
    return pool, mgr, ids


def _decode(pool, mgr, layer, q, L):
    from unifiedkv_b200.page16_native import page16_decode_attention
    e = mgr.page_table[(1, layer)]
    bt = torch.tensor([e.gpu_block_map], dtype=torch.int32, device=q.device)
    lens = torch.tensor([L], dtype=torch.int32, device=q.device)
    return page16_decode_attention(q, pool.k_cache[layer], pool.v_cache[layer], bt, lens, softmax_scale=128 ** -0.5,
                                   n_rep=4)


def test_offload_prefetch_roundtrip(cuda):
    pool, mgr, ids = _setup(cuda)
    q = torch.randn(1, 32, 128, device=cuda).to(torch.bfloat16)
    before = [_decode(pool, mgr, l, q, 1000) for l in range(3)]
    orig_k = pool.k_cache[:, ids].clone()
    orig_v = pool.v_cache[:, ids].clone()
    sel = [0, 1, 2, 5, 9, 10, 11, 12, 13, 40, 62]
    free0 = pool.n_free
    assert mgr.offload_sequence_blocks(1, sel)
    assert mgr._try_finalize_offload(1, force_sync=True)
    assert pool.n_free == free0 + len(sel)
    e = mgr.page_table[(1, 0)]
    assert all(e.gpu_block_map[i] == -1 for i in sel)
    from unifiedkv_b200.kv_types import OffloadState
    assert e.state == OffloadState.MIXED
    # scribble over the freed pages so stale data cannot pass the test
    for i in sel:
        pool.k_cache[:, ids[i]].fill_(7.0)
        pool.v_cache[:, ids[i]].fill_(7.0)
    assert mgr.ensure_sequence_blocks_on_gpu(1)
    e = mgr.page_table[(1, 0)]
    assert e.state == OffloadState.ON_GPU and all(b >= 0 for b in e.gpu_block_map)
    for l in range(3):
        got_k = pool.k_cache[l, e.gpu_block_map]
        got_v = pool.v_cache[l, e.gpu_block_map]
        assert torch.equal(got_k, orig_k[l]) and torch.equal(got_v, orig_v[l])
        assert torch.equal(_decode(pool, mgr, l, q, 1000), before[l])
    torch.cuda.synchronize()
    mgr._reclaim_slots()
    assert len(mgr._free_slots) == 128
    st = mgr.get_stats()
    assert st["offload_success"] == 1 and st["prefetch_success"] == 1


def test_reserve_decode_slot_and_release(cuda):
    pool, mgr, ids = _setup(cuda, L=32)
    n0 = pool.n_free
    assert mgr.reserve_decode_slot(1).ok  # 32 % 16 == 0 -> one new page for all layers
    assert pool.n_free == n0 - 1 and len(mgr.page_table[(1, 2)].gpu_block_map) == 3
    mgr.commit_decode_token(1)
    assert mgr.reserve_decode_slot(1).ok and pool.n_free == n0 - 1  # 33 % 16 != 0
    assert mgr.offload_sequence_blocks(1, [0])
    mgr._try_finalize_offload(1, force_sync=True)
    r = mgr.reserve_decode_slot(1)
    assert not r.ok and r.retryable and "not_on_gpu" in r.reason
    mgr.release_sequence(1)
    assert pool.n_free == 300 and len(mgr._free_slots) == 128 and not mgr.page_table
