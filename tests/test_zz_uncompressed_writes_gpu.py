"""The uncompressed page writes: PagedKVPool.write_kv_to_blocks
(core/pool.py:127-142) and the "too_short" / "input_le_budget" writeback of
the selection engine (core/scheduler.py:666-700), both the compaction
kernel's copy mode (k_blocks < 0: token p of the source -> slot p).

Reference semantics, restated in torch here: page i of ``block_ids`` receives
tokens [16 i, min(16 i + 16, seq_len)); slots past seq_len in the last page
and pages past the sequence keep their contents.  Bit-exact.  The file name
sorts last so a run that stops at the first failure has already run every
other test.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _reference_write(kc, vc, layer, block_ids, K, V):
    """core/pool.py:127-142 as written: page by page, only the rows the sequence has."""
    seq_len = K.shape[1]
    for i, bid in enumerate(block_ids):
        s, e = 16 * i, min(16 * i + 16, seq_len)
        if e > s:
            kc[layer, bid, :e - s] = K[:, s:e].transpose(0, 1)
            vc[layer, bid, :e - s] = V[:, s:e].transpose(0, 1)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("seq_len,n_ids", [(40, 3), (48, 3), (1, 1), (70, 2), (33, 5)])
def test_write_kv_to_blocks_matches_reference(cuda, dtype, seq_len, n_ids):
    from unifiedkv_b200.pool import PagedKVPool
    h_kv, d, layers = 2, 64, 3
    pool = PagedKVPool(16, layers, h_kv, d, dtype, device=cuda, n_total=20)
    g = torch.Generator(device=cuda).manual_seed(seq_len * 7 + n_ids)
    pool.k_cache.copy_(torch.randn(pool.k_cache.shape, generator=g, device=cuda).to(dtype))  # stale contents
    pool.v_cache.copy_(torch.randn(pool.v_cache.shape, generator=g, device=cuda).to(dtype))
    ref_k, ref_v = pool.k_cache.clone(), pool.v_cache.clone()
    K = torch.randn(h_kv, seq_len, d, generator=g, device=cuda).to(dtype)
    V = torch.randn(h_kv, seq_len, d, generator=g, device=cuda).to(dtype)
    ids = [int(x) for x in torch.randperm(20, generator=torch.Generator().manual_seed(n_ids))[:n_ids]]
    pool.write_kv_to_blocks(1, ids, K, V)
    _reference_write(ref_k, ref_v, 1, ids, K, V)
    torch.cuda.synchronize()
    assert torch.equal(pool.k_cache, ref_k) and torch.equal(pool.v_cache, ref_v)
    k_back, v_back = pool.read_kv_from_blocks(1, ids, seq_len)
    n = min(seq_len, 16 * n_ids)
    assert torch.equal(k_back, K[:, :n]) and torch.equal(v_back, V[:, :n])


def test_too_short_writeback_copies_the_sequence(cuda):
    """A sequence shorter than sink + obs + one block is written back whole
    (mode "too_short", effective_len = L) into fresh pages of every layer."""
    from oracle import compress as oc
    from unifiedkv_b200.pool import PagedKVPool
    from unifiedkv_b200.selection import SelectionEngine
    layers, h_kv, d, L = 2, 2, 64, 40
    pool = PagedKVPool(16, layers, h_kv, d, torch.bfloat16, device=cuda, n_total=50)
    eng = SelectionEngine(pool, num_q_heads=8, sink_len=16, obs_len=16, retain_ratio=0.25)
    k, eff_ref, mode = oc.selection_budget_blocks(L, 16, 16, 0, 0.25)
    assert mode == "too_short" and eff_ref == L
    rng = np.random.default_rng(5)
    raw = {l: tuple(torch.from_numpy(rng.standard_normal((h_kv, L, d)).astype(np.float32)).to(cuda, torch.bfloat16)
                    for _ in range(2)) for l in range(layers)}
    for l in range(layers):
        eng.q_cache[l][3] = torch.randn(8, L, d, device=cuda).to(torch.bfloat16)
    ids, selected, eff = eng.select_and_writeback(3, raw)
    torch.cuda.synchronize()
    assert eff == L and len(ids) == 3 and all(selected[l] == [] for l in range(layers))
    for l in range(layers):
        K, V = raw[l]
        kb, vb = pool.read_kv_from_blocks(l, ids, L)
        assert torch.equal(kb, K) and torch.equal(vb, V)
    assert eng.page_table[(3, 1)].seq_len == L
