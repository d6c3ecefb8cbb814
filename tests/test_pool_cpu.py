"""CPU tests of the pool bookkeeping that the decode path relies on: the FIFO
free list and watermarks of PagedKVPool (core/pool.py:95-124) and the 0-padded
int32 block table (core/pool.py:174-189).  The pool's page tensors are created
lazily, so a CPU-device pool exercises the allocator without a GPU."""
import torch

from unifiedkv_b200.pool import PagedKVPool, block_table_tensor


def test_allocator_is_fifo_and_all_or_nothing():
    pool = PagedKVPool(16, 2, 8, 128, torch.bfloat16, device="cpu", n_total=10)
    assert pool.allocate_blocks(3) == [0, 1, 2]
    assert pool.allocate_blocks(8) == []  # not enough: nothing taken
    assert pool.n_free == 7
    pool.free_blocks_by_ids([1])
    assert pool.allocate_blocks(6) == [3, 4, 5, 6, 7, 8]
    assert pool.allocate_blocks(2) == [9, 1]  # freed pages go to the back of the list
    assert pool.n_free == 0


def test_watermarks_follow_the_reference_rule():
    pool = PagedKVPool(16, 2, 8, 128, torch.bfloat16, device="cpu", n_total=100)
    assert (pool.N_wm_low, pool.N_wm_high) == (15, 40)
    assert pool.check_watermark(10) == "OK"
    pool.allocate_blocks(70)
    assert pool.check_watermark(10) == "WARNING"
    assert pool.check_watermark(31) == "VRAM_FULL"


def test_block_table_is_zero_padded_int32():
    t = block_table_tensor([[3, 4, 9], [7], []], torch.device("cpu"))
    assert t.dtype == torch.int32
    assert t.tolist() == [[3, 4, 9], [7, 0, 0], [0, 0, 0]]
    assert block_table_tensor([[], []], torch.device("cpu")).shape == (2, 0)


def test_token_writes_and_page_reads():
    """write_one_token (core/pool.py:143-152) and read_kv_from_blocks (:154-172):
    tokens written at (page, slot) read back in sequence order across pages,
    the partial last page cut at seq_len, and an empty read shaped [h_kv, 0, d]."""
    pool = PagedKVPool(16, 2, 2, 8, torch.float32, device="cpu", n_total=12)
    pages = [7, 2, 9]
    K = torch.randn(2, 40, 8)
    V = torch.randn(2, 40, 8)
    for t in range(40):
        pool.write_one_token(1, pages[t // 16], t % 16, K[:, t:t + 1], V[:, t:t + 1])
    k, v = pool.read_kv_from_blocks(1, pages, 40)
    assert k.shape == (2, 40, 8) and torch.equal(k, K) and torch.equal(v, V)
    k, v = pool.read_kv_from_blocks(1, pages, 20)
    assert torch.equal(k, K[:, :20]) and torch.equal(v, V[:, :20])
    assert torch.count_nonzero(pool.k_cache[0]) == 0  # the other layer is untouched
    k, v = pool.read_kv_from_blocks(1, [], 5)
    assert k.shape == (2, 0, 8) and v.shape == (2, 0, 8)


def test_build_cu_seqlens():
    """core/varlen.py:12-16: int32 [0, l0, l0+l1, ...]; zero-length sequences keep their slot."""
    from unifiedkv_b200.varlen import build_cu_seqlens
    cu = build_cu_seqlens([3, 0, 5, 1], "cpu")
    assert cu.dtype == torch.int32 and cu.tolist() == [0, 3, 3, 8, 9]
    assert build_cu_seqlens([], "cpu").tolist() == [0]
