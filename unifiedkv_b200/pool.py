"""Paged KV pool: ``k_cache``/``v_cache`` of shape [num_layers, N_total, 16, h_kv, d].

Mirrors ``PagedKVPool`` (core/pool.py:7-189): same constructor arguments,
sizing rule, FIFO free list, watermarks and helper methods.  Differences, all
additive: an explicit ``device`` and ``n_total`` override (the reference sizes
from ``torch.cuda.memory_allocated`` of device 0 only), page writes/reads run
through libbpkv.so kernels, and ``build_block_table`` issues one host->device
copy per table instead of one per row.
"""
from __future__ import annotations

import threading
from typing import Dict, List, Optional, Tuple

import numpy as np
import torch

from . import _lib


class PagedKVPool:
    def __init__(self, block_size: int, num_layers: int, num_kv_heads: int, head_dim: int,
                 dtype: torch.dtype = torch.float16, gpu_mem_frac: float = 0.75, cpu_mem_gb: float = 48.0,
                 *, device: Optional[torch.device] = None, n_total: Optional[int] = None):
        if int(block_size) != 16:
            raise RuntimeError(f"page16_native_shape_unsupported:block_size_{block_size}")
        self.B = int(block_size)
        self.num_layers = int(num_layers)
        self.num_kv_heads = int(num_kv_heads)
        self.head_dim = int(head_dim)
        self.dtype = dtype
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        if n_total is None:
            # core/pool.py:36-45: fraction of (total - allocated - 10% reserve)
            total = torch.cuda.get_device_properties(self.device).total_memory
            used = torch.cuda.memory_allocated(self.device)
            available = total - used - int(0.10 * total)
            max_kv_mem = int(available * gpu_mem_frac)
            elem = torch.empty((), dtype=dtype).element_size()
            bytes_per_block = 2 * self.num_layers * self.B * self.num_kv_heads * self.head_dim * elem
            n_total = max(1, max_kv_mem // bytes_per_block)
        self.N_total = int(n_total)
        self._k_cache: Optional[torch.Tensor] = None
        self._v_cache: Optional[torch.Tensor] = None
        self.lock = threading.Lock()
        self.free_blocks: List[int] = list(range(self.N_total))
        self.used_blocks: Dict[int, int] = {}
        self.cpu_budget = int(cpu_mem_gb * 1024 ** 3)
        self.cpu_used_bytes = 0
        self.N_wm_low = max(1, int(0.15 * self.N_total))
        self.N_wm_high = max(2, int(0.40 * self.N_total))

    # ---- storage -----------------------------------------------------------
    @property
    def is_allocated(self) -> bool:
        return self._k_cache is not None and self._v_cache is not None

    def ensure_allocated(self) -> None:
        if self.is_allocated:
            return
        shape = (self.num_layers, self.N_total, self.B, self.num_kv_heads, self.head_dim)
        self._k_cache = torch.zeros(shape, dtype=self.dtype, device=self.device)
        self._v_cache = torch.zeros_like(self._k_cache)

    @property
    def k_cache(self) -> torch.Tensor:
        self.ensure_allocated()
        return self._k_cache

    @property
    def v_cache(self) -> torch.Tensor:
        self.ensure_allocated()
        return self._v_cache

    def release_if_empty(self) -> bool:
        with self.lock:
            empty = len(self.used_blocks) == 0
        if not empty or not self.is_allocated:
            return False
        self._k_cache = None
        self._v_cache = None
        torch.cuda.empty_cache()
        return True

    # ---- free list (core/pool.py:94-125) ------------------------------------
    @property
    def n_free(self) -> int:
        with self.lock:
            return len(self.free_blocks)

    def allocate_blocks(self, n: int) -> List[int]:
        with self.lock:
            if len(self.free_blocks) < n:
                return []
            ids = self.free_blocks[:n]
            self.free_blocks = self.free_blocks[n:]
            for bid in ids:
                self.used_blocks[bid] = 1
            return ids

    def free_blocks_by_ids(self, block_ids: List[int]):
        with self.lock:
            for bid in block_ids:
                if bid in self.used_blocks:
                    del self.used_blocks[bid]
                self.free_blocks.append(bid)

    def check_watermark(self, n_required: int) -> str:
        with self.lock:
            n = len(self.free_blocks)
        if n < n_required:
            return "VRAM_FULL"
        if n < self.N_wm_high:
            return "WARNING"
        return "OK"

    # ---- page I/O ------------------------------------------------------------
    def _ids_tensor(self, ids: List[int]) -> torch.Tensor:
        return torch.tensor(ids, dtype=torch.int32).to(self.device, non_blocking=True)

    def write_kv_to_blocks(self, layer_id: int, block_ids: List[int], K: torch.Tensor, V: torch.Tensor):
        """K, V [h_kv, seq, d] -> pages ``block_ids`` in order (core/pool.py:127-142)."""
        seq_len = int(K.shape[1])
        n = min(len(block_ids), (seq_len + self.B - 1) // self.B)
        if n == 0:
            return
        K = K.to(self.device, self.dtype)
        V = V.to(self.device, self.dtype)
        write_pages(self.k_cache[layer_id], self.v_cache[layer_id], K, V, block_ids[:n], None, -1, 0, 0,
                    length=min(seq_len, n * self.B))

    def write_one_token(self, layer_id: int, block_id: int, pos_in_block: int, k_tok: torch.Tensor,
                        v_tok: torch.Tensor):
        self.k_cache[layer_id, block_id, pos_in_block] = k_tok.squeeze(1)
        self.v_cache[layer_id, block_id, pos_in_block] = v_tok.squeeze(1)

    def read_kv_from_blocks(self, layer_id: int, block_ids: List[int], seq_len: int) -> Tuple[torch.Tensor, torch.Tensor]:
        """Pages -> K, V [h_kv, seq_len, d] (core/pool.py:154-172); a debugging helper."""
        n = min(len(block_ids), (seq_len + self.B - 1) // self.B)
        if n == 0 or seq_len <= 0:
            e = torch.empty(self.num_kv_heads, 0, self.head_dim, dtype=self.dtype, device=self.device)
            return e, e.clone()
        ids = torch.tensor(block_ids[:n], dtype=torch.long, device=self.device)
        K = self.k_cache[layer_id].index_select(0, ids).reshape(n * self.B, self.num_kv_heads, self.head_dim)
        V = self.v_cache[layer_id].index_select(0, ids).reshape(n * self.B, self.num_kv_heads, self.head_dim)
        L = min(seq_len, n * self.B)
        return K[:L].transpose(0, 1).contiguous(), V[:L].transpose(0, 1).contiguous()

    def build_block_table(self, layer_id: int, seq_block_ids_list: List[List[int]]
                          ) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        """int32 [batch, max_blocks] table, 0-padded (core/pool.py:174-189), one H2D copy."""
        return self.k_cache[layer_id], self.v_cache[layer_id], block_table_tensor(seq_block_ids_list, self.device)


def block_table_tensor(seq_block_ids_list: List[List[int]], device: torch.device) -> torch.Tensor:
    batch = len(seq_block_ids_list)
    max_blocks = max((len(ids) for ids in seq_block_ids_list), default=0)
    host = np.zeros((batch, max(max_blocks, 1) if batch else 0), np.int32)
    for i, ids in enumerate(seq_block_ids_list):
        if ids:
            host[i, :len(ids)] = ids
    if max_blocks == 0:
        host = host[:, :0]
    t = torch.from_numpy(host)
    if device.type == "cuda":
        t = t.pin_memory().to(device, non_blocking=True)
    return t


def write_pages(k_dst: torch.Tensor, v_dst: torch.Tensor, K: torch.Tensor, V: torch.Tensor, dst_pages,
                selected: Optional[torch.Tensor], k_blocks: int, sink: int, obs: int, length: Optional[int] = None,
                dense_out: bool = False) -> None:
    """Launch bpkv_page_compact.

    k_dst/v_dst: a pool layer view [N, 16, h_kv, d] (or, with dense_out, a dense
    [h_kv, eff_len, d] tensor); K, V: [h_kv, L, d] sources; dst_pages: list or
    int32 device tensor; selected: int32 device tensor of k_blocks mid blocks,
    or [h_kv, k_blocks] with each KV head's own blocks (per-KV-head selection)
    (k_blocks < 0 = uncompressed copy of the first ``length`` tokens).
    """
    h_kv, L, d = [int(x) for x in K.shape]
    if K.stride(2) != 1 or V.stride() != K.stride():
        K = K.contiguous()
        V = V.contiguous()
    if length is not None:
        L = int(length)
    if not torch.is_tensor(dst_pages):
        dst_pages = torch.tensor(list(dst_pages), dtype=torch.int32).to(K.device, non_blocking=True)
    if dense_out:
        eff = int(k_dst.shape[1])
        ps, st, sh = 16 * d, d, eff * d
    else:
        ps, st, sh = k_dst.stride(0), k_dst.stride(1), k_dst.stride(2)
    if k_dst.dtype != K.dtype:
        raise RuntimeError("selected_writeback_shape:dtype_mismatch")
    lib = _lib.lib()  # raises page16_native_unavailable when the library is missing
    with torch.cuda.device(K.device):
        if selected is not None and selected.dim() == 2:
            if int(selected.shape[0]) != h_kv or selected.stride(1) != 1:
                raise RuntimeError("selected_writeback_shape:per_kv_head_selected")
            rc = lib.bpkv_page_compact_per_kv_head(
                K.data_ptr(), V.data_ptr(), k_dst.data_ptr(), v_dst.data_ptr(), selected.data_ptr(),
                selected.stride(0), int(k_blocks), dst_pages.data_ptr(), L, int(sink), int(obs), h_kv, d,
                K.stride(0), K.stride(1), ps, st, sh, _lib.dtype_code(K.dtype), _lib.stream_ptr(K.device))
        else:
            rc = lib.bpkv_page_compact(
                K.data_ptr(), V.data_ptr(), k_dst.data_ptr(), v_dst.data_ptr(), _lib.ptr(selected), int(k_blocks),
                dst_pages.data_ptr(), L, int(sink), int(obs), h_kv, d, K.stride(0), K.stride(1), ps, st, sh,
                _lib.dtype_code(K.dtype), _lib.stream_ptr(K.device))
    _lib.check(rc, "selected_writeback")
