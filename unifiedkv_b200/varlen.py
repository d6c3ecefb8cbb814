"""Varlen prefill attention (drop-in for core/varlen.py:1-42).

``HAS_FLASH_ATTN`` keeps the reference's flag name for importers; here it
means the native library is loaded.  The attention runs in libbpkv.so
(``bpkv_varlen_prefill``), not in flash-attn.
"""
from __future__ import annotations

from typing import List

import torch

from . import _lib

HAS_FLASH_ATTN = _lib.available()


def build_cu_seqlens(seq_lens: List[int], device="cuda") -> torch.Tensor:
    """Exclusive prefix sums [0, l0, l0+l1, ...] as int32 (core/varlen.py:12-16)."""
    cu = torch.zeros(len(seq_lens) + 1, dtype=torch.int32)
    if seq_lens:
        cu[1:] = torch.cumsum(torch.tensor([int(x) for x in seq_lens], dtype=torch.int64), 0).to(torch.int32)
    return cu.to(device)


def varlen_prefill_attention(Q: torch.Tensor, K: torch.Tensor, V: torch.Tensor, seq_lens: List[int],
                             softmax_scale: float | None = None, causal: bool = True) -> torch.Tensor:
    """Causal attention of packed sequences: Q [total, h_q, d], K/V [total, h_kv, d].

    Same call as core/varlen.py:19-42 (there: flash_attn_varlen_func with
    cu_seqlens_q == cu_seqlens_k, causal=True, scale d^-1/2).
    """
    if not _lib.available():
        raise ImportError("varlen attention requires the native library libbpkv.so")
    total, h_q, d = [int(x) for x in Q.shape]
    h_kv = int(K.shape[1])
    if K.shape != V.shape or int(K.shape[0]) != total or int(K.shape[2]) != d:
        raise RuntimeError("prefill_shape_unsupported:shape")
    if sum(int(x) for x in seq_lens) != total:
        raise RuntimeError("prefill_shape_unsupported:seq_lens")
    Q, K, V = Q.contiguous(), K.contiguous(), V.contiguous()
    out = torch.empty_like(Q)
    cu = build_cu_seqlens(seq_lens, Q.device)
    scale = float(softmax_scale) if softmax_scale is not None else d ** -0.5
    with torch.cuda.device(Q.device):
        rc = _lib.lib().bpkv_varlen_prefill(Q.data_ptr(), K.data_ptr(), V.data_ptr(), cu.data_ptr(), out.data_ptr(),
                                            len(seq_lens), h_q, h_kv, d, max(seq_lens, default=0), scale,
                                            int(bool(causal)), _lib.dtype_code(Q.dtype), _lib.stream_ptr(Q.device))
    _lib.check(rc, "varlen_prefill")
    return out
