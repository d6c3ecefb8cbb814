"""Chunked prefill into paged KV.

``paged_chunk_prefill`` is the new paged path: a chunk's queries attend to the
request's past pages plus the chunk itself (causal, bottom-right aligned, as
flash-attn defines it for seqlen_q < seqlen_k), reading K/V directly from the
16-token pool through the block table.  The chunk's own K/V must already be
in the pool (``append_chunk_kv``).  The reference instead grows a dense HF
DynamicCache per chunk (core/chunked_prefill.py:9-33, core/engine.py:1772-1854).

``ChunkedPrefillProcessor`` keeps the reference class (chunk loop over an HF
model and its memory estimate) for API compatibility.
"""
from __future__ import annotations

from typing import List, Optional, Tuple

import torch

from . import _lib
from .pool import write_pages


def paged_chunk_prefill(q_chunk: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                        block_table: torch.Tensor, past_lens, chunk_lens, softmax_scale: float, n_rep: int,
                        causal: bool = True, cu_seqlens_q: Optional[torch.Tensor] = None,
                        seqlens_k: Optional[torch.Tensor] = None, max_seqlen_q: Optional[int] = None) -> torch.Tensor:
    """q_chunk: [total_q, h_q, d] (chunks of all requests packed); k/v_cache: one
    layer's pool view [N, 16, h_kv, d]; block_table: int32 [B, max_blocks];
    past_lens / chunk_lens: per-request lists (or pass device tensors
    cu_seqlens_q [B+1] and seqlens_k [B] = past + chunk directly, with
    max_seqlen_q the longest chunk; it sizes the grid)."""
    total, h_q, d = [int(x) for x in q_chunk.shape]
    h_kv = int(k_cache.shape[2])
    if h_q != h_kv * int(n_rep) or int(k_cache.shape[1]) != 16 or int(k_cache.shape[3]) != d:
        raise RuntimeError("prefill_shape_unsupported:gqa")
    s = k_cache.stride()
    if s[3] != 1 or s[2] != d or s[1] != h_kv * d or v_cache.stride() != k_cache.stride():
        raise RuntimeError("prefill_shape_unsupported:cache_layout")
    dev = q_chunk.device
    B = int(block_table.shape[0])
    if cu_seqlens_q is None or seqlens_k is None:
        chunk_lens = [int(x) for x in chunk_lens]
        past_lens = [int(x) for x in past_lens]
        cu = [0]
        for c in chunk_lens:
            cu.append(cu[-1] + c)
        if cu[-1] != total:
            raise RuntimeError("prefill_shape_unsupported:chunk_lens")
        cu_seqlens_q = torch.tensor(cu, dtype=torch.int32).to(dev, non_blocking=True)
        seqlens_k = torch.tensor([p + c for p, c in zip(past_lens, chunk_lens)], dtype=torch.int32).to(dev, non_blocking=True)
        max_q = max(chunk_lens, default=0)
    else:
        max_q = int(max_seqlen_q) if max_seqlen_q is not None else total
    lib = _lib.lib()  # raises page16_native_unavailable when the library is missing
    q_chunk = q_chunk.contiguous()
    bt = block_table.to(torch.int32).contiguous()
    out = torch.empty_like(q_chunk)
    with torch.cuda.device(dev):
        rc = lib.bpkv_paged_prefill(
            q_chunk.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), bt.data_ptr(), cu_seqlens_q.data_ptr(),
            seqlens_k.data_ptr(), out.data_ptr(), B, h_q, h_kv, d, int(bt.shape[1]), int(max_q), s[0], bt.stride(0),
            float(softmax_scale), int(bool(causal)), _lib.dtype_code(q_chunk.dtype), _lib.stream_ptr(dev))
    _lib.check(rc, "paged_prefill")
    return out


def append_chunk_kv(k_cache: torch.Tensor, v_cache: torch.Tensor, k_chunk: torch.Tensor, v_chunk: torch.Tensor,
                    block_ids: List[int], past_len: int) -> None:
    """Write a chunk's K/V ([h_kv, n, d]) at token positions past_len.. of a
    request whose pages are ``block_ids`` (pool layer view)."""
    n = int(k_chunk.shape[1])
    if n == 0:
        return
    first = past_len // 16
    last = (past_len + n - 1) // 16
    off = past_len - first * 16
    if off == 0:
        write_pages(k_cache, v_cache, k_chunk, v_chunk, block_ids[first:last + 1], None, -1, 0, 0, length=n)
        return
    # unaligned start: fill the partial first page token-exactly, then whole pages
    head = min(16 - off, n)
    k_cache[block_ids[first], off:off + head] = k_chunk[:, :head].transpose(0, 1)
    v_cache[block_ids[first], off:off + head] = v_chunk[:, :head].transpose(0, 1)
    if n > head:
        write_pages(k_cache, v_cache, k_chunk[:, head:], v_chunk[:, head:], block_ids[first + 1:last + 1], None, -1,
                    0, 0, length=n - head)


class ChunkedPrefillProcessor:
    """Reference chunk loop (core/chunked_prefill.py:5-39), kept for API parity."""

    def __init__(self, chunk_size: int = 2048):
        self.chunk_size = chunk_size

    def run(self, model, input_ids: torch.Tensor, chunk_size: Optional[int] = None) -> Tuple[torch.Tensor, tuple]:
        cs = chunk_size or self.chunk_size
        past_kv = None
        out = None
        for start in range(0, input_ids.shape[1], cs):
            with torch.no_grad():
                out = model(input_ids=input_ids[:, start:start + cs], past_key_values=past_kv, use_cache=True)
            past_kv = out.past_key_values
        return out.logits[:, -1:, :], past_kv

    @staticmethod
    def estimate_peak_gb(seq_len: int, num_heads: int, head_dim: int, chunk_size: int) -> Tuple[float, float]:
        full_gb = num_heads * seq_len * seq_len * 2 / 1024 ** 3
        chunk_gb = num_heads * chunk_size * seq_len * 2 / 1024 ** 3
        return full_gb, chunk_gb
