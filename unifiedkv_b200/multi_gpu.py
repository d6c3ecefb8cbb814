"""Multi-GPU decode: request sharding and split-KV for one long sequence.

Replaces ``MultiGPUCoordinator`` (core/multi_gpu.py:7-123), which runs in one
process, shards KV *heads* across GPUs, mirrors every prefill layer and decode
token to each GPU with ``.to('cuda:i')`` copies, and never uses a collective
(multi-GPU decode falls back to dense rebuild, core/engine.py:2841-2851).

B200 design: one process per GPU (``torch.distributed``, NCCL over NVLink).
  * Requests are independent: ``shard_requests`` assigns whole requests to
    ranks, balanced by page count; each rank owns a pool and decodes its own
    requests.  No collective on the data path.
  * One very long sequence: ``split_pages`` gives each rank a contiguous range
    of the sequence's pages; each rank runs Page16 decode on its range with
    ``lse_out``, and the ranks exchange the [rows, d] partials plus [rows] lse
    and merge them by log-sum-exp.  ``PeerMerge`` does the exchange over NVLink
    peer memory in one kernel (each rank stores its partial straight into every
    other rank's buffer as 16-byte words that carry the call number, then polls
    the words the other ranks stored into its own buffer and merges; no fence,
    flag or collective); without it one NCCL all-gather of packed partials
    feeds the merge kernel.
The constructor arguments and the calls of the reference coordinator are kept
(register, append, evict, watermark, release); KV-head sharding is not (Page16
needs all heads of a page on one GPU), so a request lives whole on its owner rank.
"""
from __future__ import annotations

import ctypes
import heapq
from typing import Callable, Dict, List, Optional, Sequence, Tuple

import torch
import torch.distributed as dist

from . import _lib
from .pool import PagedKVPool


def shard_requests(lengths: Sequence[int], world: int) -> List[int]:
    """Owner rank of every request: longest-processing-time-first over page
    counts (deterministic: ties by request index, then lowest rank)."""
    pages = [(-((int(l) + 15) // 16), i) for i, l in enumerate(lengths)]
    pages.sort()
    heap = [(0, r) for r in range(world)]
    owner = [0] * len(lengths)
    for neg_p, i in pages:
        load, r = heapq.heappop(heap)
        owner[i] = r
        heapq.heappush(heap, (load - neg_p, r))
    return owner


def split_pages(n_pages: int, world: int) -> List[Tuple[int, int]]:
    """Contiguous [start, end) page ranges per rank, sizes differing by <= 1."""
    return [(r * n_pages // world, (r + 1) * n_pages // world) for r in range(world)]


def local_range_lens(total_len: int, start_page: int, end_page: int) -> int:
    """Tokens of a sequence of total_len that fall in pages [start, end)."""
    return max(0, min(total_len, 16 * end_page) - 16 * start_page)


def exchange_partials(out_part: torch.Tensor, lse_part: torch.Tensor, group=None) -> Tuple[torch.Tensor, torch.Tensor]:
    """All-gather per-rank partials: out_part fp32 [rows, d], lse fp32 [rows]
    -> ([world, rows, d], [world, rows]).  One collective: both travel packed
    in a single [rows, d+1] fp32 buffer."""
    world = dist.get_world_size(group)
    rows, d = out_part.shape
    packed = torch.cat([out_part.reshape(rows, d).float(), lse_part.reshape(rows, 1).float()], dim=1).contiguous()
    flat = torch.empty((world * rows, d + 1), dtype=torch.float32, device=packed.device)
    dist.all_gather_into_tensor(flat, packed, group=group)
    gathered = flat.view(world, rows, d + 1)
    return gathered[..., :d].contiguous(), gathered[..., d].contiguous()


def _split_decode(q, k_cache, v_cache, block_table, cache_seqlens, softmax_scale, n_rep, *, out_dtype,
                  lse_out=None, num_splits=0, bufs=None, rank=0, world=1, max_polls=0, status=None):
    """One call of bpkv_split_kv_decode_p2p on the current stream: decode of this
    rank's page range into fp32 CTA partials, then the fused combine (+ exchange
    and merge when world > 1).  Returns out [B, h_q, d] in out_dtype."""
    from .page16_native import _prepare
    q, block_table, cache_seqlens, (B, hq, hkv, d) = _prepare(q, k_cache, v_cache, block_table, cache_seqlens,
                                                              n_rep)
    out = torch.empty((B, hq, d), dtype=out_dtype, device=q.device)
    if lse_out is not None and (lse_out.dtype != torch.float32 or lse_out.numel() != B * hq
                                or not lse_out.is_contiguous()):
        raise RuntimeError("page16_native_shape_unsupported:lse_out")
    dev = q.device
    if status is None:
        status = torch.zeros(1, dtype=torch.int32, device=dev)
    L = _lib.lib()
    code = _lib.dtype_code(q.dtype)
    with torch.cuda.device(dev):
        stream = torch.cuda.current_stream(dev)
        ws = _lib.workspace_for(L.bpkv_page16_decode_workspace_size(B, hq, hkv, d, code), dev, stream, "page16")
        rc = L.bpkv_split_kv_decode_p2p(
            q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), block_table.data_ptr(), cache_seqlens.data_ptr(),
            out.data_ptr(), _lib.ptr(lse_out), B, hq, hkv, d, int(block_table.shape[1]),
            q.stride(0), q.stride(1), k_cache.stride(0), block_table.stride(0), float(softmax_scale), code,
            _lib.dtype_code(out_dtype), ws.data_ptr(), ws.numel(), int(num_splits), bufs, int(rank), int(world),
            int(max_polls), status.data_ptr(), stream.cuda_stream)
    _lib.check(rc, "split_kv_decode_p2p")
    return out


def decode_partial(q, k_cache, v_cache, block_table, cache_seqlens, softmax_scale, n_rep, num_splits=0):
    """This rank's fp32 partial of a split sequence: (out fp32 [B, h_q, d], lse fp32 [B, h_q]).
    No rounding to the cache dtype (the NCCL exchange carries it as is)."""
    B, hq = int(q.shape[0]), int(q.shape[1])
    lse = torch.empty((B, hq), dtype=torch.float32, device=q.device)
    out = _split_decode(q, k_cache, v_cache, block_table, cache_seqlens, softmax_scale, n_rep,
                        out_dtype=torch.float32, lse_out=lse, num_splits=num_splits)
    return out, lse


class PeerMerge:
    """NVLink peer-memory exchange + merge of split-KV partials.

    Collective set-up, on every rank of ``group`` with the same ``rows`` and
    ``head_dim``: the library allocates this rank's exchange buffer, the CUDA IPC
    handles travel once over the process group, and the other ranks' buffers are
    mapped into this process.  Then ``decode`` (bpkv_split_kv_decode_p2p: decode,
    fp32 combine, exchange and merge in two launches) or ``merge``
    (bpkv_split_kv_merge_p2p, for a partial the caller already holds) is called on
    every rank in the same order; the call count lives in device memory, so calls
    captured in a CUDA graph replay correctly.  ``close`` (collective) unmaps and
    frees.

    A wait for a peer's words that runs out sets a device status word and writes
    NaN rows; ``check()`` reads the status (a host synchronisation), clears it and
    raises, and ``check=True`` on a call does that right after it.
    """

    def __init__(self, rows: int, head_dim: int, group=None, device: Optional[torch.device] = None,
                 max_polls: int = 1 << 22):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.rows, self.head_dim = int(rows), int(head_dim)
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        self.max_polls = int(max_polls)
        L = _lib.lib()
        nbytes = L.bpkv_peer_exchange_bytes(self.world, self.rows, self.head_dim)
        if nbytes == 0:
            raise RuntimeError(f"peer_exchange_shape:world_{self.world}_rows_{rows}_head_dim_{head_dim}")
        own = ctypes.c_void_p()
        handle = ctypes.create_string_buffer(64)
        with torch.cuda.device(self.device):
            _lib.check(L.bpkv_peer_buffer_alloc(nbytes, ctypes.byref(own), handle), "peer_exchange_alloc")
        self._own = own.value
        handles: List[bytes] = [b""] * self.world
        dist.all_gather_object(handles, handle.raw, group=group)
        self._opened: List[int] = []
        bufs = []
        with torch.cuda.device(self.device):
            for r, h in enumerate(handles):
                if r == self.rank:
                    bufs.append(self._own)
                    continue
                p = ctypes.c_void_p()
                _lib.check(L.bpkv_peer_buffer_open(h, ctypes.byref(p)), "peer_exchange_open")
                self._opened.append(p.value)
                bufs.append(p.value)
        self._bufs = (ctypes.c_void_p * self.world)(*bufs)
        self.status = torch.zeros(1, dtype=torch.int32, device=self.device)

    def decode(self, q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, block_table: torch.Tensor,
               cache_seqlens: torch.Tensor, softmax_scale: float, n_rep: int, lse_out: Optional[torch.Tensor] = None,
               num_splits: int = 0, check: bool = False) -> torch.Tensor:
        """Split-KV decode of this rank's page range, merged with every other rank's
        range: q [B, h_q, d] (identical on all ranks, B * h_q == rows) -> [B, h_q, d]
        in q's dtype, on every rank."""
        B, hq, d = [int(x) for x in q.shape]
        if B * hq != self.rows or d != self.head_dim:
            raise RuntimeError("peer_exchange_shape:decode")
        out = _split_decode(q, k_cache, v_cache, block_table, cache_seqlens, softmax_scale, n_rep,
                            out_dtype=q.dtype, lse_out=lse_out, num_splits=num_splits, bufs=self._bufs,
                            rank=self.rank, world=self.world, max_polls=self.max_polls, status=self.status)
        if check:
            self.check()
        return out

    def merge(self, part_out: torch.Tensor, part_lse: torch.Tensor, out_dtype: Optional[torch.dtype] = None,
              lse_out: Optional[torch.Tensor] = None, check: bool = False) -> torch.Tensor:
        """part_out [rows, d] (fp32/fp16/bf16, this rank's partial), part_lse fp32 [rows]
        -> merged [rows, d] in out_dtype (default: part_out's dtype)."""
        rows, d = int(part_out.shape[0]), int(part_out.shape[1])
        if rows != self.rows or d != self.head_dim:
            raise RuntimeError("peer_exchange_shape:merge")
        out_dtype = out_dtype or part_out.dtype
        part_out = part_out.contiguous()
        part_lse = part_lse.reshape(rows).float().contiguous()
        out = torch.empty((rows, d), dtype=out_dtype, device=part_out.device)
        with torch.cuda.device(self.device):
            rc = _lib.lib().bpkv_split_kv_merge_p2p(
                part_out.data_ptr(), part_lse.data_ptr(), self._bufs, self.rank, self.world, rows, d,
                self.max_polls, out.data_ptr(), _lib.ptr(lse_out), self.status.data_ptr(),
                _lib.dtype_code(part_out.dtype), _lib.dtype_code(out_dtype), _lib.stream_ptr(self.device))
        _lib.check(rc, "split_kv_merge_p2p")
        if check:
            self.check()
        return out

    def check(self) -> None:
        """Host check of the device status (synchronises): raises if a wait ran out
        since the last check; the status is cleared either way."""
        st = int(self.status.item())
        if st != 0:
            self.status.zero_()
            raise RuntimeError("peer_exchange_timeout: a rank's partial did not arrive")

    def close(self) -> None:
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)  # no rank still stores into a buffer that is about to go
        L = _lib.lib()
        with torch.cuda.device(self.device):
            for p in self._opened:
                _lib.check(L.bpkv_peer_buffer_close(p), "peer_exchange_close")
            self._opened = []
        dist.barrier(group=self.group)
        with torch.cuda.device(self.device):
            if self._own is not None:
                _lib.check(L.bpkv_peer_buffer_free(self._own), "peer_exchange_free")
                self._own = None


def _native_merge(parts: torch.Tensor, lses: torch.Tensor, out_dtype: torch.dtype):
    from .page16_native import lse_combine
    return lse_combine(parts, lses, out_dtype, return_lse=True)


def split_kv_decode(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, local_block_table: torch.Tensor,
                    local_lens: torch.Tensor, softmax_scale: float, n_rep: int, group=None,
                    merge: Optional[Callable] = None, peer: Optional[PeerMerge] = None,
                    num_splits: int = 0) -> torch.Tensor:
    """Decode one (or a few) sequences whose pages are split across ranks.

    Each rank passes q (identical on all ranks, [B, h_q, d]), its own pool
    view, the block table of ITS page range and the token count in that range.
    Returns the merged [B, h_q, d] output (q's dtype) on every rank.  A rank
    whose range is empty contributes lse = -inf (nothing).  Every partial stays
    fp32 until the final merge.  With ``peer`` (a PeerMerge for rows = B*h_q) the
    partials travel over NVLink peer memory, combined, exchanged and merged in
    one kernel after the decode; without it one NCCL all-gather of the packed
    fp32 partials feeds the merge kernel.
    """
    B, hq, d = [int(x) for x in q.shape]
    if peer is not None:
        return peer.decode(q, k_cache, v_cache, local_block_table, local_lens, softmax_scale, n_rep,
                           num_splits=num_splits)
    part, lse = decode_partial(q, k_cache, v_cache, local_block_table, local_lens, softmax_scale, n_rep,
                               num_splits=num_splits)
    parts, lses = exchange_partials(part.reshape(B * hq, d), lse.reshape(B * hq), group)
    merge = merge or _native_merge
    out, _ = merge(parts, lses, q.dtype)
    return out.reshape(B, hq, d)


class MultiGPUCoordinator:
    """Per-rank coordinator (one process per GPU).

    Keeps the reference constructor signature (core/multi_gpu.py:8-47); the
    pool of this rank holds ALL KV heads (``num_kv_heads_total``) and the
    requests this rank owns.
    """

    def __init__(self, num_gpus: int, block_size: int, num_layers: int, num_kv_heads_total: int, head_dim: int,
                 dtype: torch.dtype = torch.float16, cpu_mem_gb_per_gpu: float = 16.0, *, group=None,
                 n_pages: Optional[int] = None, device: Optional[torch.device] = None):
        self.group = group
        self.distributed = dist.is_available() and dist.is_initialized()
        self.world = dist.get_world_size(group) if self.distributed else 1
        self.rank = dist.get_rank(group) if self.distributed else 0
        if int(num_gpus) != self.world:
            raise RuntimeError(f"multi_gpu_world_mismatch num_gpus={num_gpus} world={self.world}")
        self.num_gpus = int(num_gpus)
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        self.pool = PagedKVPool(block_size, num_layers, num_kv_heads_total, head_dim, dtype,
                                gpu_mem_frac=0.9, cpu_mem_gb=cpu_mem_gb_per_gpu, device=self.device, n_total=n_pages)
        self.owner: Dict[int, int] = {}
        self.local_blocks: Dict[int, List[int]] = {}
        self.seq_lens: Dict[Tuple[int, int], int] = {}  # (seq, layer) -> tokens stored on this rank
        self.offloader = None  # optional, with the engine's evict_coldest_sequence policy

    def assign(self, seq_lens: Dict[int, int]) -> Dict[int, int]:
        """Shard new requests {seq_id: length} over ranks; returns {seq_id: rank}."""
        ids = sorted(seq_lens)
        owners = shard_requests([seq_lens[i] for i in ids], self.world)
        for sid, r in zip(ids, owners):
            self.owner[sid] = r
        return {sid: self.owner[sid] for sid in ids}

    def is_local(self, seq_id: int) -> bool:
        return self.owner.get(int(seq_id), 0) == self.rank

    def allocate(self, seq_id: int, n_blocks: int) -> List[int]:
        if not self.is_local(seq_id):
            raise RuntimeError(f"multi_gpu_not_owner seq={seq_id} rank={self.rank}")
        ids = self.pool.allocate_blocks(n_blocks)
        if not ids:
            raise MemoryError(f"Cannot allocate {n_blocks} blocks for seq={seq_id} on rank {self.rank}")
        self.local_blocks.setdefault(int(seq_id), []).extend(ids)
        return ids

    def _split_kv_heads(self, K: torch.Tensor, V: torch.Tensor) -> List[Tuple[torch.Tensor, torch.Tensor]]:
        """The reference cuts K/V [h_kv_total, ...] into per-GPU head ranges
        (core/multi_gpu.py:49-59); a rank here holds every head of its own
        requests, so there is one shard: all heads."""
        return [(K.contiguous(), V.contiguous())]

    def register_layer_from_full_kv(self, seq_id: int, layer_id: int, K: torch.Tensor, V: torch.Tensor) -> bool:
        """One layer of a prefilled sequence, K/V [h_kv_total, L, d] (core/multi_gpu.py:76-84).

        Only the owning rank stores it; the first layer registered allocates the
        ceil(L/16) pages that every layer of the sequence shares.  Returns
        whether this rank stored it."""
        if not self.is_local(seq_id):
            return False
        L = int(K.shape[1])
        need = (L + self.pool.B - 1) // self.pool.B
        ids = self.local_blocks.get(int(seq_id))
        if ids is None:
            ids = self.allocate(seq_id, need)
        elif len(ids) < need:
            raise RuntimeError(f"multi_gpu_layer_len_mismatch seq={seq_id} layer={layer_id} len={L} pages={len(ids)}")
        self.pool.write_kv_to_blocks(int(layer_id), list(ids), K, V)
        self.seq_lens[(int(seq_id), int(layer_id))] = L
        return True

    def register_all_gpus(self, seq_id: int, layer_id: int, kv_shards: List[Tuple[torch.Tensor, torch.Tensor]]) -> bool:
        """The reference's per-GPU head shards of one layer (core/multi_gpu.py:61-74),
        put back together: this rank's pool holds every head."""
        K = torch.cat([k for k, _ in kv_shards], dim=0)
        V = torch.cat([v for _, v in kv_shards], dim=0)
        return self.register_layer_from_full_kv(seq_id, layer_id, K, V)

    def append_decode_token_all_gpus(self, seq_id: int, layer_id: int, k_tok: torch.Tensor,
                                     v_tok: torch.Tensor) -> bool:
        """This step's token of one layer, k_tok/v_tok [h_kv_total, 1, d]
        (core/multi_gpu.py:86-102).  The owning rank stores it at position
        seq_len of that layer; layer 0 takes a new page (shared by all layers)
        when the last one is full, as core/offload.py:926-951 does.  Returns
        whether this rank stored it."""
        if not self.is_local(seq_id):
            return False
        key = (int(seq_id), int(layer_id))
        n = self.seq_lens.get(key, 0)
        ids = self.local_blocks.get(int(seq_id), [])
        if n >= len(ids) * self.pool.B:
            if int(layer_id) != 0:
                raise RuntimeError(f"multi_gpu_append_without_page seq={seq_id} layer={layer_id}")
            self.allocate(seq_id, 1)
            ids = self.local_blocks[int(seq_id)]
        self.pool.write_one_token(int(layer_id), ids[n // self.pool.B], n % self.pool.B, k_tok, v_tok)
        self.seq_lens[key] = n + 1
        return True

    def global_evict(self, current_layer: int, current_seq: int) -> None:
        """Ask this rank's offloader to evict its coldest sequence (core/multi_gpu.py:104-110);
        the world-wide view is each rank doing the same.  No offloader with a
        policy: nothing to evict."""
        del current_layer
        evict = getattr(self.offloader, "evict_coldest_sequence", None)
        if evict is None:
            return
        try:
            evict(current_seq)
        except MemoryError:
            pass

    def global_watermark(self) -> str:
        """Worst free ratio over ranks (core/multi_gpu.py:112-119 thresholds)."""
        ratio = self.pool.n_free / max(1, self.pool.N_total)
        if self.distributed and self.world > 1:
            dev = self.device if dist.get_backend(self.group) == "nccl" else torch.device("cpu")
            t = torch.tensor([ratio], dtype=torch.float64, device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MIN, group=self.group)
            ratio = float(t.item())
        if ratio < 0.15:
            return "VRAM_FULL"
        if ratio < 0.35:
            return "WARNING"
        return "OK"

    def release_all(self, seq_id: int) -> None:
        ids = self.local_blocks.pop(int(seq_id), None)
        if ids:
            self.pool.free_blocks_by_ids(ids)
        self.owner.pop(int(seq_id), None)
        for key in [k for k in self.seq_lens if k[0] == int(seq_id)]:
            del self.seq_lens[key]
