"""Pinned-host offload and prefetch of pool pages, batched and asynchronous.

Replaces the transfer mechanism of ``AsyncOffloadManager`` (core/offload.py:547-757):
there, every (page, layer, K/V) is one small ``copy_`` into a freshly pinned
host tensor, and ``ensure_sequence_blocks_on_gpu`` synchronises the host
before decode (core/offload.py:752).  Here:
  * host memory is one pinned arena of fixed-size slots allocated once; a slot
    holds one logical page of one sequence for ALL layers, K and V;
  * an offload gathers the selected pages of every layer into a device
    staging buffer with one ``bpkv_page_gather`` launch per K/V (the pool is
    addressed as a flat [L*N] page array), then one device->host copy, all on
    a low-priority side stream, completed by a CUDA event;
  * a prefetch is the mirror image (one host->device copy, one
    ``bpkv_page_scatter`` per K/V); ``ensure_sequence_blocks_on_gpu`` makes the
    compute stream wait on the prefetch event instead of blocking the host.
The page-table bookkeeping keeps the reference's names and states
(``BlockTableEntry.gpu_block_map`` with -1 for host-resident pages,
``OffloadState``, ``_try_finalize_offload/prefetch``, stats counters).  The
pressure policy that picks victims (P2) is out of scope.
"""
from __future__ import annotations

import threading
from typing import Dict, List, Optional, Tuple

import torch

from . import _lib
from .kv_types import BlockTableEntry, DecodeAppendResult, OffloadState
from .pool import PagedKVPool


class AsyncOffloadManager:
    def __init__(self, pool: PagedKVPool, num_layers: int, host_slots: int = 0, staging_pages: int = 512):
        self.pool = pool
        self.num_layers = int(num_layers)
        self.lock = threading.Lock()
        self.page_table: Dict[Tuple[int, int], BlockTableEntry] = {}
        self.device = pool.device
        self.transfer_stream = torch.cuda.Stream(device=self.device, priority=-1)
        self.page_elems = 16 * pool.num_kv_heads * pool.head_dim
        self.staging_pages = int(staging_pages)
        self.host_slots = int(host_slots) if host_slots else max(1, pool.N_total // 4)
        self._arena: Optional[torch.Tensor] = None    # pinned [2, slots, L, page_elems]
        self._staging: Optional[torch.Tensor] = None  # device [2, staging_pages, L, page_elems]
        self._free_slots: List[int] = list(range(self.host_slots))
        self._slot_of: Dict[Tuple[int, int], int] = {}  # (seq, logical page) -> host slot
        self._pending: Dict[int, dict] = {}  # seq -> in-flight transfer
        self._stats: Dict[str, int] = {}

    # ---- helpers -------------------------------------------------------------
    def _inc_stat(self, key: str, inc: int = 1):
        self._stats[key] = self._stats.get(key, 0) + int(inc)

    def get_stats(self, reset: bool = False) -> Dict[str, int]:
        out = dict(self._stats)
        if reset:
            self._stats.clear()
        return out

    def _ensure_buffers(self):
        if self._arena is None:
            self._arena = torch.empty((2, self.host_slots, self.num_layers, self.page_elems), dtype=self.pool.dtype,
                                      pin_memory=True)
        if self._staging is None:
            self._staging = torch.empty((2, self.staging_pages, self.num_layers, self.page_elems),
                                        dtype=self.pool.dtype, device=self.device)

    @staticmethod
    def _ensure_entry_maps(entry: BlockTableEntry):
        n = len(entry.block_ids)
        if len(entry.gpu_block_map) != n:
            entry.gpu_block_map = list(entry.block_ids)
        if len(entry.cpu_k_blocks) != n:
            entry.cpu_k_blocks = [None] * n
            entry.cpu_v_blocks = [None] * n

    @staticmethod
    def _update_entry_state(entry: BlockTableEntry):
        on_gpu = sum(1 for b in entry.gpu_block_map if int(b) >= 0)
        if on_gpu == len(entry.gpu_block_map):
            entry.state = OffloadState.ON_GPU
        elif on_gpu == 0:
            entry.state = OffloadState.ON_CPU
        else:
            entry.state = OffloadState.MIXED

    def _entries(self, seq_id: int) -> List[BlockTableEntry]:
        return [self.page_table[(seq_id, l)] for l in range(self.num_layers) if (seq_id, l) in self.page_table]

    def register_sequence(self, seq_id: int, block_ids: List[int], seq_len: int) -> None:
        """Page-table rows for a sequence whose pages (shared by all layers) are already written."""
        with self.lock:
            for l in range(self.num_layers):
                self.page_table[(int(seq_id), l)] = BlockTableEntry(
                    seq_id=int(seq_id), layer_id=l, state=OffloadState.ON_GPU, block_ids=list(block_ids),
                    seq_len=int(seq_len), logical_seq_len=int(seq_len), materialized_blocks=len(block_ids),
                    gpu_block_map=list(block_ids), cpu_k_blocks=[None] * len(block_ids),
                    cpu_v_blocks=[None] * len(block_ids))

    def register(self, seq_id: int, layer_id: int, K: torch.Tensor, V: torch.Tensor) -> List[int]:
        """One layer of a prefilled sequence, K/V [h_kv, L, d], into fresh pages
        (core/offload.py:451-473).  Returns the page ids."""
        seq_len = int(K.shape[1])
        n_blocks = (seq_len + self.pool.B - 1) // self.pool.B
        block_ids = self.pool.allocate_blocks(n_blocks)
        if not block_ids:
            raise MemoryError(f"GPU blocks exhausted: seq={seq_id} layer={layer_id}")
        self.pool.write_kv_to_blocks(int(layer_id), block_ids, K, V)
        with self.lock:
            self.page_table[(int(seq_id), int(layer_id))] = BlockTableEntry(
                seq_id=int(seq_id), layer_id=int(layer_id), state=OffloadState.ON_GPU, block_ids=list(block_ids),
                seq_len=seq_len, logical_seq_len=seq_len, materialized_blocks=len(block_ids),
                gpu_block_map=list(block_ids), cpu_k_blocks=[None] * n_blocks, cpu_v_blocks=[None] * n_blocks)
        return list(block_ids)

    def register_all_layers(self, seq_id: int, block_ids: List[int], seq_len: int, K_list: list, V_list: list,
                            anchor_k_means: Optional[list] = None, logical_seq_len: Optional[int] = None) -> None:
        """Every layer of a sequence into the same, already allocated pages
        (core/offload.py:475-510); a layer whose K is None is skipped."""
        logical = int(seq_len if logical_seq_len is None else logical_seq_len)
        for layer_id, (K, V) in enumerate(zip(K_list, V_list)):
            if K is None:
                continue
            anchor = anchor_k_means[layer_id] if anchor_k_means is not None and layer_id < len(anchor_k_means) else None
            if torch.is_tensor(anchor):
                anchor = anchor.detach().cpu()
            self.pool.write_kv_to_blocks(layer_id, list(block_ids), K, V)
            with self.lock:
                self.page_table[(int(seq_id), layer_id)] = BlockTableEntry(
                    seq_id=int(seq_id), layer_id=layer_id, state=OffloadState.ON_GPU, block_ids=list(block_ids),
                    seq_len=int(seq_len), logical_seq_len=logical, materialized_blocks=len(block_ids),
                    prefill_anchor_k_mean=anchor, gpu_block_map=list(block_ids),
                    cpu_k_blocks=[None] * len(block_ids), cpu_v_blocks=[None] * len(block_ids))

    def _sequence_has_state(self, seq_id: int, state: OffloadState) -> bool:
        return any(e.state == state for e in self._entries(seq_id))

    def get_sequence_residency(self, seq_id: int) -> Dict[str, int]:
        """Residency summary with the reference's keys (core/offload.py:307-360).
        No residency-protection policy runs here, so residency_protected is 0."""
        entries = self._entries(seq_id)
        if not entries:
            return dict(exists=0, on_gpu=0, resident_blocks=0, logical_blocks=0, materialized_blocks=0,
                        resident_ratio_x1000=0, has_cpu_blocks=0, state_mixed=0, last_access=-1,
                        residency_protected=0)
        resident = logical = materialized = 0
        on_gpu = has_cpu = mixed = 0
        last_access = -1
        for e in entries:
            self._ensure_entry_maps(e)
            resident = max(resident, sum(1 for b in e.gpu_block_map if int(b) >= 0))
            materialized = max(materialized, int(e.materialized_blocks or len(e.gpu_block_map)))
            n_tok = int(e.logical_seq_len or e.seq_len or 0)
            logical = max(logical, (n_tok + self.pool.B - 1) // self.pool.B)
            on_gpu |= int(e.state == OffloadState.ON_GPU)
            mixed |= int(e.state == OffloadState.MIXED)
            has_cpu |= int(any(x is not None for x in e.cpu_k_blocks))
            last_access = max(last_access, int(getattr(e, "last_access", -1)))
        return dict(exists=1, on_gpu=on_gpu, resident_blocks=resident, logical_blocks=logical,
                    materialized_blocks=materialized,
                    resident_ratio_x1000=int(1000 * resident / max(1, materialized)) if materialized > 0 else 0,
                    has_cpu_blocks=has_cpu, state_mixed=mixed, last_access=last_access, residency_protected=0)

    def _flat_ids(self, pages: List[int]) -> torch.Tensor:
        """Flat [L*N] pool page indices, page-major: entry j*L + l is page j of layer l."""
        N = self.pool.N_total
        ids = [l * N + p for p in pages for l in range(self.num_layers)]
        return torch.tensor(ids, dtype=torch.int32).pin_memory().to(self.device, non_blocking=True)

    def _move(self, gather: bool, flat_ids: torch.Tensor, which: int) -> None:
        """Pool pages <-> staging[which][:n] ([n, L, page_elems]) on the transfer stream."""
        cache = self.pool.k_cache if which == 0 else self.pool.v_cache
        stage = self._staging[which]
        n = int(flat_ids.numel())
        lib = _lib.lib()
        code = _lib.dtype_code(self.pool.dtype)
        st = self.transfer_stream.cuda_stream
        if gather:
            rc = lib.bpkv_page_gather(cache.data_ptr(), flat_ids.data_ptr(), n, stage.data_ptr(), self.page_elems,
                                      self.page_elems, code, st)
        else:
            rc = lib.bpkv_page_scatter(stage.data_ptr(), flat_ids.data_ptr(), n, cache.data_ptr(), self.page_elems,
                                       self.page_elems, code, st)
        _lib.check(rc, "page_gather" if gather else "page_scatter")

    def _alloc_slots(self, n: int) -> Optional[List[int]]:
        """n host slots, lowest-first (sorted free list keeps batches mostly contiguous)."""
        if len(self._free_slots) < n:
            return None
        self._free_slots.sort()
        out, self._free_slots = self._free_slots[:n], self._free_slots[n:]
        return out

    @staticmethod
    def _runs(slots: List[int]) -> List[Tuple[int, int, int]]:
        """(first batch index, first slot, length) of each contiguous slot run."""
        runs = []
        i = 0
        while i < len(slots):
            j = i
            while j + 1 < len(slots) and slots[j + 1] == slots[j] + 1:
                j += 1
            runs.append((i, slots[i], j - i + 1))
            i = j + 1
        return runs

    # ---- offload (device -> pinned host) -----------------------------------
    def offload_sequence_blocks(self, seq_id: int, logical_block_indices: List[int]) -> bool:
        """Start copying the given logical pages (all layers, K and V) of a
        sequence to host slots; pool pages are freed when the copy completes
        (``_try_finalize_offload``).  Mirrors core/offload.py:547-599."""
        self._inc_stat('offload_calls')
        self._try_finalize_offload(seq_id, force_sync=False)
        self._try_finalize_prefetch(seq_id, force_sync=False)
        if seq_id in self._pending:
            self._inc_stat('offload_fail')
            return False
        entries = self._entries(seq_id)
        if not entries or any(e.state not in (OffloadState.ON_GPU, OffloadState.MIXED) for e in entries):
            self._inc_stat('offload_fail')
            return False
        first = entries[0]
        self._ensure_entry_maps(first)
        sel = sorted({int(i) for i in logical_block_indices
                      if 0 <= int(i) < len(first.gpu_block_map) and int(first.gpu_block_map[int(i)]) >= 0})
        if not sel:
            self._inc_stat('offload_fail')
            return False
        self._ensure_buffers()
        slots = self._alloc_slots(len(sel))
        if slots is None:
            self._inc_stat('offload_fail')
            return False
        pages = [int(first.gpu_block_map[i]) for i in sel]
        ts = self.transfer_stream
        ts.wait_stream(torch.cuda.current_stream(self.device))  # pages may still be written by compute
        with torch.cuda.stream(ts):
            for c0 in range(0, len(sel), self.staging_pages):
                chunk = pages[c0:c0 + self.staging_pages]
                ids = self._flat_ids(chunk)
                for w in (0, 1):
                    self._move(True, ids, w)
                    for i, s0, n in self._runs(slots[c0:c0 + len(chunk)]):
                        self._arena[w, s0:s0 + n].copy_(self._staging[w, i:i + n], non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(ts)
        self._pending[seq_id] = dict(kind="offload", event=ev, sel=sel, pages=pages, slots=slots)
        for e in entries:
            e.state = OffloadState.OFFLOAD_INFLIGHT
            e.transfer_event = ev
            e.pending_block_indices = list(sel)
        self._inc_stat('offload_blocks', len(sel))
        return True

    def offload_sequence(self, seq_id: int) -> bool:
        entries = self._entries(seq_id)
        if not entries:
            self._inc_stat('offload_fail')
            return False
        return self.offload_sequence_blocks(seq_id, list(range(len(entries[0].gpu_block_map))))

    def _try_finalize_offload(self, seq_id: int, force_sync: bool = False) -> bool:
        p = self._pending.get(seq_id)
        if p is None or p["kind"] != "offload":
            return False
        if not force_sync and not p["event"].query():
            return False
        p["event"].synchronize()
        del self._pending[seq_id]
        for e in self._entries(seq_id):
            self._ensure_entry_maps(e)
            for idx, slot in zip(p["sel"], p["slots"]):
                e.gpu_block_map[idx] = -1
                e.cpu_k_blocks[idx] = ("host_slot", slot)
                e.cpu_v_blocks[idx] = ("host_slot", slot)
            e.transfer_event = None
            e.pending_block_indices = None
            self._update_entry_state(e)
        for idx, slot in zip(p["sel"], p["slots"]):
            self._slot_of[(seq_id, idx)] = slot
        self.pool.free_blocks_by_ids(p["pages"])
        self.pool.cpu_used_bytes += len(p["sel"]) * 2 * self.num_layers * self.page_elems * self.pool.k_cache.element_size()
        self._inc_stat('offload_success')
        return True

    # ---- prefetch (pinned host -> device) ------------------------------------
    def _host_resident(self, seq_id: int, logical_block_indices: List[int]) -> List[int]:
        """The requested logical pages that live in host slots, ascending."""
        entries = self._entries(seq_id)
        if not entries:
            return []
        first = entries[0]
        return sorted({int(i) for i in logical_block_indices
                       if 0 <= int(i) < len(first.gpu_block_map) and int(first.gpu_block_map[int(i)]) < 0
                       and (seq_id, int(i)) in self._slot_of})

    def prefetch_sequence(self, seq_id: int) -> bool:
        """Every host-resident page of the sequence back to the pool
        (core/offload.py:693-706); waits for the copy if it could not finish at once."""
        entries = self._entries(seq_id)
        if not entries:
            self._inc_stat("prefetch_noop")
            self._inc_stat("prefetch_success")
            return True
        n = max(len(e.gpu_block_map) for e in entries)
        ok = self.prefetch_sequence_blocks(seq_id, list(range(n)))
        if not ok:
            ok = self._try_finalize_prefetch(seq_id, force_sync=True)
        return bool(ok)

    def ensure_sequence_on_gpu(self, seq_id: int, allow_evict: bool = True,
                               protected_seqs: Optional[List[int]] = None) -> bool:
        """All pages of the sequence resident (core/offload.py:759-778)."""
        entries = self._entries(seq_id)
        if not entries:
            self._inc_stat("ensure_fail")
            return False
        n = max(len(e.gpu_block_map) for e in entries)
        return self.ensure_sequence_blocks_on_gpu(seq_id, list(range(n)), allow_evict=allow_evict,
                                                  protected_seqs=protected_seqs)

    def prefetch_sequence_blocks(self, seq_id: int, logical_block_indices: List[int]) -> bool:
        """Start copying host-resident pages back into fresh pool pages.  Returns
        True when nothing is left to fetch, False while a transfer is in flight
        or on failure (core/offload.py:620-691)."""
        self._inc_stat('prefetch_calls')
        if self._try_finalize_prefetch(seq_id, force_sync=False):
            return True
        if seq_id in self._pending:
            self._inc_stat('prefetch_inflight')
            return False
        entries = self._entries(seq_id)
        if not entries:
            self._inc_stat('prefetch_noop')
            return True
        sel = self._host_resident(seq_id, logical_block_indices)
        if not sel:
            self._inc_stat('prefetch_noop')
            return True
        pages = self.pool.allocate_blocks(len(sel))
        if len(pages) != len(sel):
            self._inc_stat('prefetch_fail')
            return False
        slots = [self._slot_of[(seq_id, i)] for i in sel]
        ts = self.transfer_stream
        ts.wait_stream(torch.cuda.current_stream(self.device))  # new pages may still be read by compute
        with torch.cuda.stream(ts):
            for c0 in range(0, len(sel), self.staging_pages):
                chunk = pages[c0:c0 + self.staging_pages]
                ids = self._flat_ids(chunk)
                for w in (0, 1):
                    for i, s0, n in self._runs(slots[c0:c0 + len(chunk)]):
                        self._staging[w, i:i + n].copy_(self._arena[w, s0:s0 + n], non_blocking=True)
                    self._move(False, ids, w)
            ev = torch.cuda.Event()
            ev.record(ts)
        self._pending[seq_id] = dict(kind="prefetch", event=ev, sel=sel, pages=pages, slots=slots)
        for e in entries:
            e.state = OffloadState.PREFETCH_INFLIGHT
            e.transfer_event = ev
            e.pending_block_indices = list(sel)
        self._inc_stat('prefetch_blocks', len(sel))
        return False

    def _apply_prefetch(self, seq_id: int, p: dict) -> None:
        del self._pending[seq_id]
        for e in self._entries(seq_id):
            for idx, page in zip(p["sel"], p["pages"]):
                e.gpu_block_map[idx] = int(page)
                e.block_ids[idx] = int(page)
                e.cpu_k_blocks[idx] = None
                e.cpu_v_blocks[idx] = None
            e.transfer_event = None
            e.pending_block_indices = None
            self._update_entry_state(e)
        for idx in p["sel"]:
            self._slot_of.pop((seq_id, idx), None)
        self._free_slots.extend(p["slots"])
        self.pool.cpu_used_bytes = max(0, self.pool.cpu_used_bytes - len(p["sel"]) * 2 * self.num_layers *
                                       self.page_elems * self.pool.k_cache.element_size())
        self._inc_stat('prefetch_success')

    def _try_finalize_prefetch(self, seq_id: int, force_sync: bool = False) -> bool:
        p = self._pending.get(seq_id)
        if p is None or p["kind"] != "prefetch":
            return False
        if not force_sync and not p["event"].query():
            return False
        p["event"].synchronize()
        # host slots are reusable only once the H2D copy has read them
        self._apply_prefetch(seq_id, p)
        return True

    def ensure_sequence_blocks_on_gpu(self, seq_id: int, missing_block_indices: Optional[List[int]] = None,
                                      allow_evict: bool = True, protected_seqs: Optional[List[int]] = None,
                                      stream: Optional[torch.cuda.Stream] = None) -> bool:
        """Make the given pages resident for work queued on ``stream`` (default:
        the current stream) WITHOUT blocking the host: the prefetch runs on the
        side stream and ``stream`` waits on its event.  Host slots are recycled
        when the event has completed (polled by later calls).  Parameters as in
        core/offload.py:708-757: with ``allow_evict``, a pool short of pages
        first evicts other sequences through the engine's policy (if one is
        attached; ``protected_seqs`` and this sequence are never chosen)."""
        self._inc_stat("ensure_calls")
        self._try_finalize_offload(seq_id, force_sync=True)
        entries = self._entries(seq_id)
        if not entries:
            return False
        idx = list(range(len(entries[0].gpu_block_map))) if missing_block_indices is None else missing_block_indices
        if allow_evict and seq_id not in self._pending:
            need = len(self._host_resident(seq_id, idx))
            if need > self.pool.n_free:
                self._evict_until_free(need, seq_id, protected_seqs=[int(seq_id)] + list(protected_seqs or []))
        if self.prefetch_sequence_blocks(seq_id, idx):
            return True
        p = self._pending.get(seq_id)
        if p is None or p["kind"] != "prefetch":
            return False
        (stream or torch.cuda.current_stream(self.device)).wait_event(p["event"])
        # the mapping is valid in stream order from here on; only slot reuse waits for the event
        slots_event = p["event"]
        self._apply_prefetch(seq_id, dict(p, slots=[]))
        self._deferred_slots = getattr(self, "_deferred_slots", [])
        self._deferred_slots.append((slots_event, p["slots"]))
        self._reclaim_slots()
        return True

    def _reclaim_slots(self) -> None:
        keep = []
        for ev, slots in getattr(self, "_deferred_slots", []):
            if ev.query():
                self._free_slots.extend(slots)
            else:
                keep.append((ev, slots))
        self._deferred_slots = keep

    # ---- decode bookkeeping (core/offload.py:780-866) -------------------------
    def _evict_until_free(self, target_free: int, exclude_seq: int,
                          protected_seqs: Optional[List[int]] = None) -> bool:
        """Free pool pages by evicting whole sequences until ``target_free`` pages are
        free (core/offload.py:257-287).  The victim choice is the engine's pressure
        policy, supplied as ``evict_coldest_sequence(exclude_seq, protected_seqs=...)``
        (returns the victim's id after starting its offload; raises MemoryError when
        nothing can go); without one, nothing can be evicted."""
        evict = getattr(self, "evict_coldest_sequence", None)
        target = max(0, int(target_free))
        while self.pool.n_free < target:
            if evict is None:
                return False
            before = int(self.pool.n_free)
            try:
                victim = evict(exclude_seq, protected_seqs=protected_seqs)
            except MemoryError:
                return False
            try:
                self._try_finalize_offload(int(victim), force_sync=True)
            except Exception:
                return False
            if int(self.pool.n_free) <= before and int(self.pool.n_free) < target:
                self._inc_stat("evict_fail")
                return False
        return True

    def _decode_fail(self, retryable: bool, reason: str) -> DecodeAppendResult:
        self._inc_stat("decode_append_fail")
        if retryable:
            self._inc_stat("decode_append_retryable")
        return DecodeAppendResult(ok=False, retryable=retryable, reason=reason)

    def reserve_decode_slot(self, seq_id: int) -> DecodeAppendResult:
        """Make room for one decode token of a fully resident sequence: a new page
        (the same id in every layer) when the last page is full.  Same checks,
        order, reasons and stats as the reference."""
        entries = [self.page_table.get((seq_id, l)) for l in range(self.num_layers)]
        if any(e is None for e in entries):
            return self._decode_fail(False, f"missing_page_table_entry seq={seq_id}")
        for e in entries:
            self._ensure_entry_maps(e)
            if e.state != OffloadState.ON_GPU:
                return self._decode_fail(True, f"direct_decode_not_on_gpu seq={seq_id} state={e.state}")
            if any(int(b) < 0 for b in e.gpu_block_map):
                return self._decode_fail(True, f"direct_decode_resident_missing seq={seq_id}")
            if not e.block_ids:
                self._inc_stat("decode_append_fail")
                return DecodeAppendResult(ok=False, retryable=True, reason=f"direct_decode_no_gpu_blocks seq={seq_id}")
        seq_len = int(entries[0].seq_len)
        if any(int(e.seq_len) != seq_len for e in entries):
            return self._decode_fail(False, f"direct_decode_inconsistent_seq_len seq={seq_id}")
        if seq_len % self.pool.B == 0:
            new = self.pool.allocate_blocks(1)
            if not new:
                if not self._evict_until_free(max(self.pool.N_wm_high, 1), seq_id, protected_seqs=[seq_id]):
                    return self._decode_fail(True, "direct_decode_expand_evict_failed")
                new = self.pool.allocate_blocks(1)
                if not new:
                    return self._decode_fail(True, "direct_decode_expand_alloc_failed")
            for e in entries:
                self._ensure_entry_maps(e)
                e.block_ids.append(int(new[0]))
                e.gpu_block_map.append(int(new[0]))
                e.cpu_k_blocks.append(None)
                e.cpu_v_blocks.append(None)
                e.materialized_blocks = len(e.gpu_block_map)
                self._update_entry_state(e)
        return DecodeAppendResult(ok=True)

    def append_decode_token(self, seq_id: int, layer_id: int, k_tok: torch.Tensor,
                            v_tok: torch.Tensor) -> DecodeAppendResult:
        """Store one layer's decode token, k_tok/v_tok [h_kv, 1, d], at position
        seq_len of that layer (core/offload.py:868-960): a non-resident sequence is
        brought back first, layer 0 takes a new page (for every layer) when the
        last one is full.  Same reasons and stats as the reference.  The batched
        decode path uses reserve_decode_slot + the fused append of the decode
        launch instead."""
        self._inc_stat("decode_append_calls")
        key = (int(seq_id), int(layer_id))
        entry = self.page_table.get(key)
        if entry is None:
            return self._decode_fail(False, f"missing_page_table_entry seq={seq_id} layer={layer_id}")
        self._ensure_entry_maps(entry)
        if entry.state != OffloadState.ON_GPU or any(int(b) < 0 for b in entry.gpu_block_map):
            # True from ensure means the page map is valid in stream order (the copy may still run)
            ok = self.ensure_sequence_on_gpu(seq_id, allow_evict=True, protected_seqs=[seq_id])
            if not ok or any(int(b) < 0 for b in entry.gpu_block_map):
                reason = f"prefetch_before_decode_append_failed seq={seq_id}"
                if self._sequence_has_state(seq_id, OffloadState.PREFETCH_INFLIGHT):
                    reason = f"prefetch_inflight seq={seq_id}"
                elif self._sequence_has_state(seq_id, OffloadState.OFFLOAD_INFLIGHT):
                    reason = f"offload_inflight seq={seq_id}"
                return self._decode_fail(True, reason)
            entry = self.page_table.get(key)
            if entry is None:
                return self._decode_fail(False, f"missing_page_table_after_prefetch seq={seq_id} layer={layer_id}")
        self._ensure_entry_maps(entry)
        if not entry.block_ids:
            self._inc_stat("decode_append_fail")
            return DecodeAppendResult(ok=False, retryable=True,
                                      reason=f"no_gpu_blocks_for_decode_append seq={seq_id} layer={layer_id}")
        last_used = int(entry.seq_len) % self.pool.B
        if last_used == 0 and int(layer_id) == 0:
            new = self.pool.allocate_blocks(1)
            if not new:
                if not self._evict_until_free(max(self.pool.N_wm_high, 1), seq_id, protected_seqs=[seq_id]):
                    return self._decode_fail(True, "decode_expand_evict_failed")
                new = self.pool.allocate_blocks(1)
                if not new:
                    return self._decode_fail(True, "decode_expand_alloc_failed")
            for e in self._entries(seq_id):
                self._ensure_entry_maps(e)
                e.block_ids.append(int(new[0]))
                e.gpu_block_map.append(int(new[0]))
                e.cpu_k_blocks.append(None)
                e.cpu_v_blocks.append(None)
                e.materialized_blocks = len(e.gpu_block_map)
                self._update_entry_state(e)
        self.pool.write_one_token(int(layer_id), int(entry.block_ids[-1]), last_used, k_tok, v_tok)
        if int(entry.logical_seq_len or 0) <= 0:
            entry.logical_seq_len = int(entry.seq_len)
        entry.seq_len += 1
        entry.logical_seq_len += 1
        entry.materialized_blocks = max(int(entry.materialized_blocks or 0), len(entry.gpu_block_map))
        self._inc_stat("decode_append_success")
        return DecodeAppendResult(ok=True)

    def commit_decode_token(self, seq_id: int) -> None:
        for e in self._entries(seq_id):
            e.seq_len += 1
            e.logical_seq_len = int(e.logical_seq_len or e.seq_len - 1) + 1

    def release_sequence(self, seq_id: int):
        self._try_finalize_offload(seq_id, force_sync=True)
        self._try_finalize_prefetch(seq_id, force_sync=True)
        entries = self._entries(seq_id)
        if entries:
            self.pool.free_blocks_by_ids([int(b) for b in entries[0].gpu_block_map if int(b) >= 0])
        for key in [k for k in self._slot_of if k[0] == seq_id]:
            self._free_slots.append(self._slot_of.pop(key))
        for l in range(self.num_layers):
            self.page_table.pop((seq_id, l), None)
