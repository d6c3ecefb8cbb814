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
