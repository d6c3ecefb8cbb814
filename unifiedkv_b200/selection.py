"""Selected-writeback compression path of the scheduler, on libbpkv.so kernels.

Mirrors the KVScheduler methods of core/scheduler.py:547-878 with the same
names, arguments, return values and error strings, so a drop-in either mixes
``SelectedWritebackOps`` into a scheduler or uses ``SelectionEngine`` below:

  _selection_budget_blocks(L)                      scheduler.py:547-564
  _score_layer_blocks_for_selection(K, Q_obs)      scheduler.py:565-592
  _compute_per_layer_selected_blocks(seq, raw)     scheduler.py:594-639
  _allocate_writeback_blocks(seq, n)               scheduler.py:654-664
  _write_block_indexed_layer_to_pool(...)          scheduler.py:702-733
  _write_selected_layer_to_pool(...)               scheduler.py:735-799
  _selected_writeback_transaction(...)             scheduler.py:805-878

Differences: scoring never materialises the [h_q, W, T] attention matrix; the
top-k breaks ties by the lowest block index; the writeback of every layer is
one compaction kernel; ``select_and_writeback`` runs all layers with selected
indices kept on the device and a single device->host copy at the end (the
reference syncs once per layer).
"""
from __future__ import annotations

import math
import os
from typing import Dict, List, Optional, Tuple

import torch

from .compress import SMOOTH_IF_3, BlockAlignedSnapKV, block_scores, topk_blocks
from .kv_types import BlockTableEntry, OffloadState
from .pool import PagedKVPool, write_pages


def _env_flag(name: str) -> bool:
    return str(os.environ.get(name, "")).strip().lower() in {"1", "true", "yes", "on"}


class SelectedWritebackOps:
    """Requires: self.snapkv (BlockAlignedSnapKV), self.pool (PagedKVPool),
    self.n_rep, self.head_dim, self.num_layers, self.q_cache[layer][seq] (Q of
    the prefill, [h_q, L, d]), self.page_table dict, self.writeback_transaction_rollbacks."""

    # ---- budget ----------------------------------------------------------
    def _selection_budget_blocks(self, L: int) -> Tuple[int, int, str]:
        B = int(self.snapkv.B)
        budget = int(getattr(self.snapkv, "retain_budget_tokens", 0) or 0)
        Ls, Lo = int(self.snapkv.Ls), int(self.snapkv.Lo)
        if budget > 0 and int(L) <= budget:
            return 0, int(L), "input_le_budget"
        if int(L) < Ls + Lo + B:
            return 0, int(L), "too_short"
        mid_blocks = int(math.ceil(max(0, int(L) - Ls - Lo) / B))
        if budget > 0:
            k = max(0, min(mid_blocks, int(math.floor(max(0, budget - Ls - Lo) / B))))
            return int(k), Ls + k * B + Lo, "fixed_budget"
        k = max(1, min(mid_blocks, int(math.floor(float(self.snapkv.retain_ratio) * mid_blocks))))
        return int(k), Ls + k * B + Lo, "ratio"

    # ---- scoring -----------------------------------------------------------
    def _score_layer_blocks_for_selection(self, K: torch.Tensor, Q_obs: torch.Tensor) -> torch.Tensor:
        if K.dim() != 3 or Q_obs.dim() != 3:
            raise RuntimeError("selected_writeback_bad_score_shape")
        dev = self.pool.device
        K = K if K.device == dev else K.to(dev)
        Q_obs = Q_obs if Q_obs.device == dev else Q_obs.to(dev)
        if Q_obs.dtype != K.dtype:
            Q_obs = Q_obs.to(K.dtype)
        L = int(K.shape[1])
        if L < int(self.snapkv.Ls) + int(self.snapkv.Lo) + int(self.snapkv.B):
            return torch.empty((0,), dtype=torch.float32, device=dev)
        self.score_full_attention_materialized = 0
        return block_scores(K, Q_obs, int(self.snapkv.Ls), int(self.snapkv.Lo), float(self.head_dim) ** -0.5,
                            SMOOTH_IF_3, per_kv_head=bool(getattr(self.snapkv, "per_kv_head", False)))

    def _select_layer_device(self, layer_id: int, seq_id: int, raw, k_blocks: int) -> torch.Tensor:
        Q_full = self.q_cache[layer_id].get(seq_id)
        if Q_full is None:
            raise RuntimeError(f"selected_writeback_missing_q seq={seq_id} layer={layer_id}")
        Q_obs = Q_full[:, -int(self.snapkv.Lo):, :]
        score = self._score_layer_blocks_for_selection(raw[0], Q_obs)
        n = int(score.shape[-1]) if score.dim() >= 1 else 0
        return topk_blocks(score, max(0, min(int(k_blocks), n)))

    def _compute_per_layer_selected_blocks(self, seq_id: int, raw_by_layer) -> Tuple[Dict[int, List[int]], int, int, str]:
        first = next((kv for kv in raw_by_layer.values() if kv is not None), None)
        if first is None:
            raise RuntimeError(f"selected_writeback_missing_raw seq={seq_id}")
        L = int(first[0].shape[1])
        k_blocks, effective_len, mode = self._selection_budget_blocks(L)
        selected: Dict[int, List[int]] = {}
        if k_blocks <= 0 or mode in ("input_le_budget", "too_short"):
            selected = {int(l): [] for l in range(self.num_layers)}
        else:
            dev_sel = []
            for layer_id in range(self.num_layers):
                raw = raw_by_layer.get(layer_id)
                if raw is None:
                    raise RuntimeError(f"selected_writeback_missing_raw seq={seq_id} layer={layer_id}")
                dev_sel.append(self._select_layer_device(layer_id, seq_id, raw, k_blocks))
            host = [t.cpu().tolist() for t in dev_sel]  # one sync point per sequence
            selected = {int(l): host[l] for l in range(self.num_layers)}  # [k] or per KV head [h_kv][k]
        self._record_selection_debug(L, k_blocks, effective_len, mode, selected)
        return selected, int(effective_len), int(L), str(mode)

    def _record_selection_debug(self, L, k_blocks, effective_len, mode, selected):
        total_blocks = int(math.ceil(max(1, int(effective_len)) / int(self.pool.B)))
        self.selected_global_block_count = total_blocks
        self.writeback_block_selection_shared_layers = 0
        budget = int(getattr(self.snapkv, "retain_budget_tokens", 0) or 0)
        self.snapkv.last_debug = {
            "block_size": int(self.snapkv.B), "sink_len": int(self.snapkv.Ls), "obs_len": int(self.snapkv.Lo),
            "retain_ratio": float(self.snapkv.retain_ratio), "retain_budget_tokens": budget,
            "compression_mode": "fixed_budget" if budget > 0 else "ratio", "logical_seq_len": int(L),
            "retained_block_count": int(k_blocks), "selected_global_block_count": total_blocks,
            "effective_retained_tokens": int(effective_len),
            "retained_block_idx": [selected.get(int(l), []) for l in range(self.num_layers)],
            "shared_block_selection": False, "selection_granularity": "per_layer_block_topk",
            "selection_scope": "per_kv_head" if getattr(self.snapkv, "per_kv_head", False) else "shared",
            "compression_skipped": mode if mode in ("input_le_budget", "too_short") else "",
        }

    # ---- allocation ----------------------------------------------------------
    def _allocate_writeback_blocks(self, seq_id: int, n_req: int) -> List[int]:
        evict = getattr(self, "_evict_one_for_prefill_allocation", None)
        if evict is not None:
            if self.pool.n_free < self.pool.N_wm_low:
                target = max(int(n_req), int(self.pool.N_wm_high))
                while self.pool.n_free < target:
                    evict(seq_id, target)
            while self.pool.n_free < int(n_req):
                evict(seq_id, int(n_req))
        ids = self.pool.allocate_blocks(int(n_req))
        if not ids:
            raise MemoryError(f"Cannot allocate {int(n_req)} blocks for seq={seq_id}")
        return list(ids)

    # ---- writeback -------------------------------------------------------------
    def _write_block_indexed_layer_to_pool(self, layer_id: int, block_ids: List[int], K: torch.Tensor,
                                           V: torch.Tensor, source_block_indices: List[int]) -> bool:
        """Aligned fast path: page i <- source block source_block_indices[i]."""
        B = int(self.pool.B)
        if not source_block_indices or len(source_block_indices) != len(block_ids):
            return False
        if int(K.shape[1]) % B != 0 or int(V.shape[1]) % B != 0:
            return False
        raw_blocks = int(K.shape[1]) // B
        mx = max(int(x) for x in source_block_indices)
        if min(int(x) for x in source_block_indices) < 0 or mx >= raw_blocks:
            return False
        dev = self.pool.device
        K = K.to(dev, self.pool.dtype)
        V = V.to(dev, self.pool.dtype)
        # express "page i <- block s_i" as a compaction with sink=obs=0
        sel = torch.tensor([int(x) for x in source_block_indices], dtype=torch.int32).to(dev, non_blocking=True)
        write_pages(self.pool.k_cache[layer_id], self.pool.v_cache[layer_id], K, V, block_ids, sel,
                    len(source_block_indices), 0, 0)
        return True

    def _write_selected_layer_to_pool(self, layer_id: int, block_ids: List[int], K: torch.Tensor, V: torch.Tensor,
                                      selected_mid_blocks, effective_len: int, mode: str):
        L = int(K.shape[1])
        Ls, Lo = int(self.snapkv.Ls), int(self.snapkv.Lo)
        anchor_tokens = max(0, int(min(self.pool.B, Lo)))
        a0 = max(0, L - Lo)
        a1 = min(L, a0 + anchor_tokens)
        anchor = K[:, a0:a1, :].float().mean(dim=(0, 1)).detach() if a1 > a0 else None
        dev = self.pool.device
        K = K.to(dev, self.pool.dtype)
        V = V.to(dev, self.pool.dtype)
        kc, vc = self.pool.k_cache[layer_id], self.pool.v_cache[layer_id]
        if mode in ("input_le_budget", "too_short"):
            write_pages(kc, vc, K, V, block_ids, None, -1, 0, 0, length=int(effective_len))
            return anchor
        if torch.is_tensor(selected_mid_blocks):
            sel = selected_mid_blocks.to(dev, torch.int32).contiguous()
        else:  # [k] shared, or [h_kv][k] per KV head
            sel = torch.tensor(selected_mid_blocks, dtype=torch.int32).to(dev, non_blocking=True)
        k = int(sel.shape[-1]) if sel.dim() >= 1 else 0
        if Ls + 16 * k + Lo != int(effective_len):
            raise RuntimeError(f"selected_writeback_len_mismatch got={Ls + 16 * k + Lo} expected={effective_len}")
        write_pages(kc, vc, K, V, block_ids, sel, k, Ls, Lo)
        return anchor

    def _selected_writeback_transaction(self, seq_id: int, raw_by_layer, selected_mid_blocks_by_layer,
                                        effective_len: int, logical_len: int, mode: str,
                                        backend: str = "gpu_selected_writeback") -> None:
        n_req = int(math.ceil(max(1, int(effective_len)) / int(self.pool.B)))
        block_ids = self._allocate_writeback_blocks(seq_id, n_req)
        entries: Dict[Tuple[int, int], BlockTableEntry] = {}
        try:
            if backend == "gpu_selected_writeback" and _env_flag("KV_MIDDLEWARE_FORCE_GPU_WRITEBACK_OOM"):
                raise torch.cuda.OutOfMemoryError("forced selected writeback OOM")
            anchors = {}
            for layer_id in range(self.num_layers):
                raw = raw_by_layer.get(layer_id)
                if raw is None:
                    raise RuntimeError(f"selected_writeback_missing_raw seq={seq_id} layer={layer_id}")
                sel = (selected_mid_blocks_by_layer.get(int(layer_id), [])
                       if isinstance(selected_mid_blocks_by_layer, dict) else selected_mid_blocks_by_layer)
                anchors[layer_id] = self._write_selected_layer_to_pool(layer_id, block_ids, raw[0], raw[1], sel,
                                                                       int(effective_len), mode)
            for layer_id in range(self.num_layers):
                a = anchors.get(layer_id)
                entries[(int(seq_id), int(layer_id))] = BlockTableEntry(
                    seq_id=int(seq_id), layer_id=int(layer_id), state=OffloadState.ON_GPU, block_ids=list(block_ids),
                    seq_len=int(effective_len), logical_seq_len=int(logical_len),
                    materialized_blocks=len(block_ids),
                    prefill_anchor_k_mean=a.cpu() if torch.is_tensor(a) else a,
                    gpu_block_map=list(block_ids), cpu_k_blocks=[None] * len(block_ids),
                    cpu_v_blocks=[None] * len(block_ids))
            self.page_table.update(entries)
        except Exception:
            self.writeback_transaction_rollbacks = getattr(self, "writeback_transaction_rollbacks", 0) + 1
            try:
                self.pool.free_blocks_by_ids(block_ids)
            except Exception:
                pass
            raise

    # ---- fused all-layer path -------------------------------------------------------
    def select_and_writeback(self, seq_id: int, raw_by_layer) -> Tuple[List[int], Dict[int, List[int]], int]:
        """Score, select and compact every layer of one sequence with the selected
        indices kept on the device; one device->host copy at the end.
        Returns (block_ids, selected_by_layer, effective_len)."""
        first = next((kv for kv in raw_by_layer.values() if kv is not None), None)
        if first is None:
            raise RuntimeError(f"selected_writeback_missing_raw seq={seq_id}")
        L = int(first[0].shape[1])
        k_blocks, eff, mode = self._selection_budget_blocks(L)
        dev_sel = {}
        if k_blocks > 0 and mode not in ("input_le_budget", "too_short"):
            for layer_id in range(self.num_layers):
                dev_sel[layer_id] = self._select_layer_device(layer_id, seq_id, raw_by_layer[layer_id], k_blocks)
        self._selected_writeback_transaction(seq_id, raw_by_layer, dev_sel, eff, L, mode)
        host = {l: t.cpu().tolist() for l, t in dev_sel.items()}
        selected = {l: host.get(l, []) for l in range(self.num_layers)}
        self._record_selection_debug(L, k_blocks, eff, mode, selected)
        return self.page_table[(int(seq_id), 0)].block_ids, selected, eff


class SelectionEngine(SelectedWritebackOps):
    """Minimal scheduler state for the selected-writeback path: a pool, the
    compressor settings, cached window queries and a page table."""

    def __init__(self, pool: PagedKVPool, num_q_heads: int, sink_len: int = 16, obs_len: int = 16,
                 retain_ratio: float = 0.2, retain_budget_tokens: int = 0, per_kv_head: bool = False):
        self.pool = pool
        self.num_layers = pool.num_layers
        self.num_kv_heads = pool.num_kv_heads
        self.head_dim = pool.head_dim
        self.num_q_heads = int(num_q_heads)
        self.n_rep = self.num_q_heads // self.num_kv_heads
        self.snapkv = BlockAlignedSnapKV(16, sink_len, obs_len, retain_ratio, retain_budget_tokens,
                                         per_kv_head=per_kv_head)
        self.q_cache: List[Dict[int, torch.Tensor]] = [dict() for _ in range(self.num_layers)]
        self.page_table: Dict[Tuple[int, int], BlockTableEntry] = {}
        self.writeback_transaction_rollbacks = 0
        self.selected_global_block_count = 0

    def release_sequence(self, seq_id: int) -> None:
        ids = None
        for l in range(self.num_layers):
            e = self.page_table.pop((int(seq_id), l), None)
            if e is not None and ids is None:
                ids = list(e.block_ids)
        if ids:
            self.pool.free_blocks_by_ids(ids)
