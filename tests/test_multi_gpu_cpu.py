"""Multi-GPU host logic on CPU: request sharding, page splitting, and the
partial exchange + LSE merge of split-KV decode, run as world-size-2 gloo ranks.
The CUDA decode itself is replaced by the oracle on each rank's page range, so
these tests cover only the host-side plumbing (no GPU here)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle.page16 import lse_merge_reference, page16_decode_reference
from unifiedkv_b200.multi_gpu import (MultiGPUCoordinator, exchange_partials, local_range_lens, shard_requests,
                                      split_pages)


def test_shard_requests_balanced_and_deterministic():
    rng = np.random.default_rng(0)
    lens = rng.integers(4096, 32769, size=256)
    for world in (1, 2, 4, 8):
        own = shard_requests(lens, world)
        assert own == shard_requests(lens, world)
        loads = np.zeros(world)
        for l, r in zip(lens, own):
            loads[r] += (l + 15) // 16
        assert loads.max() - loads.min() <= 2048  # within one max request
        assert sorted(set(own)) == list(range(world))


def test_split_pages_cover():
    for n in (0, 1, 7, 8192):
        for w in (1, 2, 3, 8):
            r = split_pages(n, w)
            assert r[0][0] == 0 and r[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(r, r[1:]))
            assert max(e - s for s, e in r) - min(e - s for s, e in r) <= 1
    assert local_range_lens(1000, 0, 10) == 160 and local_range_lens(1000, 60, 63) == 40


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    try:
        _worker_body(rank, world, port, q)
    except Exception as exc:  # report instead of leaving the peer waiting
        q.put((rank, repr(exc), None, None))
        raise


def _worker_body(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=__import__("datetime").timedelta(seconds=60))
    try:
        rng = np.random.default_rng(5)
        L, hq, hkv, d = 1000, 8, 2, 32
        n_pages = (L + 15) // 16
        qv = rng.standard_normal((1, hq, d))
        k = rng.standard_normal((n_pages, 16, hkv, d))
        v = rng.standard_normal((n_pages, 16, hkv, d))
        s, e = split_pages(n_pages, world)[rank]
        n_local = local_range_lens(L, s, e)
        bt = np.arange(s, e, dtype=np.int32)[None]
        part, lse = page16_decode_reference(qv, k, v, bt, np.array([n_local]), d ** -0.5, hq // hkv,
                                            return_lse=True)
        parts, lses = exchange_partials(torch.from_numpy(part.reshape(hq, d)), torch.from_numpy(lse.reshape(hq)))
        merged, _ = lse_merge_reference(parts.numpy(), lses.numpy())
        full = page16_decode_reference(qv, k, v, np.arange(n_pages, dtype=np.int32)[None], np.array([L]),
                                       d ** -0.5, hq // hkv)
        err = float(np.max(np.abs(merged - full[0])))
        coord = MultiGPUCoordinator(world, 16, 2, hkv, d, torch.float32, device=torch.device("cpu"),
                                    n_pages=100 if rank == 0 else 10)
        own = coord.assign({10: 5000, 11: 300, 12: 9000})
        for sid in own:  # each rank fills 4 pages of every request it owns
            if coord.is_local(sid):
                coord.allocate(sid, 4)
        wm = coord.global_watermark()
        q.put((rank, err, own, wm))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2])
def test_split_kv_exchange_gloo(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    res.sort()
    for rank, err, own, wm in res:
        assert not isinstance(err, str), err
        assert err < 1e-6  # partials travel as fp32
        assert own == res[0][2]  # every rank computes the same assignment
    # the largest request goes to rank 0, the other two to rank 1 (LPT)
    assert res[0][2] == {10: 1, 11: 1, 12: 0}
    # rank 1 (10-page pool, 8 used) is at 20% free: every rank sees the global minimum
    assert res[0][3] == res[1][3] == "WARNING"


def test_coordinator_register_append_evict_release():
    """The reference's coordinator calls (core/multi_gpu.py:61-123) on one rank over a
    CPU pool: registration allocates the shared pages once, head shards go back
    together, decode tokens land at each layer's length with layer 0 taking the new
    page, another rank's requests are not stored, eviction reaches the offloader's
    policy, release frees everything.  The page write of a whole layer is the copy
    kernel on a GPU; a torch restatement of the reference's page loop stands in here."""
    coord = MultiGPUCoordinator(1, 16, 2, 4, 8, torch.float32, device=torch.device("cpu"), n_pages=20)
    pool = coord.pool

    def write_kv_to_blocks(layer_id, block_ids, K, V):  # core/pool.py:127-142
        for i, bid in enumerate(block_ids):
            s, e = 16 * i, min(16 * i + 16, K.shape[1])
            if e > s:
                pool.k_cache[layer_id, bid, :e - s] = K[:, s:e].transpose(0, 1)
                pool.v_cache[layer_id, bid, :e - s] = V[:, s:e].transpose(0, 1)

    pool.write_kv_to_blocks = write_kv_to_blocks
    assert coord.assign({5: 40, 6: 10}) == {5: 0, 6: 0}
    g = torch.Generator().manual_seed(0)
    K = [torch.randn(4, 40, 8, generator=g) for _ in range(2)]
    V = [torch.randn(4, 40, 8, generator=g) for _ in range(2)]
    assert coord.register_layer_from_full_kv(5, 0, K[0], V[0])
    ids = list(coord.local_blocks[5])
    assert len(ids) == 3 and pool.n_free == 17
    shards = [(K[1][:2], V[1][:2]), (K[1][2:], V[1][2:])]  # the reference's per-GPU head shards
    assert coord.register_all_gpus(5, 1, shards) and coord.local_blocks[5] == ids and pool.n_free == 17
    toks = [[(torch.randn(4, 1, 8, generator=g), torch.randn(4, 1, 8, generator=g)) for _ in range(2)]
            for _ in range(10)]
    for step in toks:  # positions 40..49: the page boundary at 48 is crossed by layer 0 first
        for layer, (kt, vt) in enumerate(step):
            assert coord.append_decode_token_all_gpus(5, layer, kt, vt)
    assert len(coord.local_blocks[5]) == 4 and pool.n_free == 16
    for layer in range(2):
        kb, vb = pool.read_kv_from_blocks(layer, coord.local_blocks[5], 50)
        want_k = torch.cat([K[layer]] + [toks[t][layer][0] for t in range(10)], dim=1)
        want_v = torch.cat([V[layer]] + [toks[t][layer][1] for t in range(10)], dim=1)
        assert torch.equal(kb, want_k) and torch.equal(vb, want_v)
        assert coord.seq_lens[(5, layer)] == 50
    # a layer other than 0 reaching a full last page first has no page to write into
    for _ in range(14):
        coord.append_decode_token_all_gpus(5, 1, *toks[0][1])
    with pytest.raises(RuntimeError, match="multi_gpu_append_without_page seq=5 layer=1"):
        coord.append_decode_token_all_gpus(5, 1, *toks[0][1])
    # another rank's request: nothing stored here
    coord.owner[7] = 1
    assert not coord.register_layer_from_full_kv(7, 0, K[0], V[0])
    assert not coord.append_decode_token_all_gpus(7, 0, *toks[0][0])
    # eviction goes to the offloader's policy; MemoryError (nothing to evict) is absorbed
    coord.global_evict(0, 5)  # no offloader: nothing happens
    calls = []

    class Off:
        def evict_coldest_sequence(self, seq):
            calls.append(seq)
            raise MemoryError

    coord.offloader = Off()
    coord.global_evict(3, 5)
    assert calls == [5]
    coord.release_all(5)
    assert pool.n_free == 20 and not any(k[0] == 5 for k in coord.seq_lens) and 5 not in coord.owner
