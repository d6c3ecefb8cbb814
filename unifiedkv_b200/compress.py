"""Block-aligned SnapKV compression on the GPU (drop-in for core/compress.py).

``BlockAlignedSnapKV`` keeps the reference's constructor, ``compress`` contract
and ``last_debug`` keys (core/compress.py:23-175).  The scoring runs in the
fused libbpkv.so kernels (no [h_q, W, T] attention matrix, no repeat_kv copy),
the top-k is deterministic with ties broken by the lowest block index (the
reference's torch.topk leaves tie order unspecified), and the gather/concat of
sink, selected mid blocks and observation tail is one compaction kernel.
"""
from __future__ import annotations

import math
from typing import Any, Dict, Tuple

import torch

from . import _lib
from .pool import write_pages

# smoothing modes of bpkv_block_score
SMOOTH_NONE, SMOOTH_IF_3, SMOOTH_ALWAYS = 0, 1, 2


def repeat_kv(x: torch.Tensor, n_rep: int) -> torch.Tensor:
    """[b, h_kv, s, d] -> [b, h_kv*n_rep, s, d] (core/compress.py:7-20).  Kept for
    API compatibility; the kernels here never materialise it."""
    if n_rep == 1:
        return x
    b, h, s, d = x.shape
    return x[:, :, None, :, :].expand(b, h, n_rep, s, d).reshape(b, h * n_rep, s, d)


def block_scores(K: torch.Tensor, Q_obs: torch.Tensor, sink_len: int, obs_len: int,
                 softmax_scale: float | None = None, smooth: int = SMOOTH_ALWAYS,
                 per_kv_head: bool = False) -> torch.Tensor:
    """Per-16-token-block scores of K_mid = K[:, sink:L-obs] (zero-padded to a
    multiple of 16) under the observation window Q_obs.

    K: [h_kv, L, d]; Q_obs: [h_q, W, d] (same dtype, bf16 or fp16, CUDA).
    Returns fp32 [N], N = ceil((L - sink - obs)/16); the math of
    core/compress.py:116-130 / core/scheduler.py:581-591.  With per_kv_head the
    max over q heads is taken within each KV group only and the result is
    fp32 [h_kv, N] (this build's addition; the reference shares one score).
    """
    if K.dim() != 3 or Q_obs.dim() != 3:
        raise RuntimeError("selected_writeback_bad_score_shape")
    h_kv, L, d = [int(x) for x in K.shape]
    h_q, W, dq = [int(x) for x in Q_obs.shape]
    if dq != d or Q_obs.dtype != K.dtype:
        raise RuntimeError("selected_writeback_bad_score_shape")
    if K.stride(2) != 1:
        K = K.contiguous()
    if Q_obs.stride(2) != 1:
        Q_obs = Q_obs.contiguous()
    scale = float(softmax_scale) if softmax_scale is not None else d ** -0.5
    n = math.ceil((L - sink_len - obs_len) / 16)
    out = torch.empty((h_kv, max(n, 0)) if per_kv_head else (max(n, 0),), dtype=torch.float32, device=K.device)
    lib = _lib.lib()
    with torch.cuda.device(K.device):
        nbytes = lib.bpkv_block_score_workspace_size(h_q, W, L, int(sink_len), int(obs_len))
        ws = _lib.workspace(nbytes, K.device, "score")
        fn = lib.bpkv_block_score_per_kv_head if per_kv_head else lib.bpkv_block_score
        rc = fn(K.data_ptr(), Q_obs.data_ptr(), out.data_ptr(), h_kv, h_q, L, W, d, int(sink_len),
                int(obs_len), K.stride(0), K.stride(1), Q_obs.stride(0), Q_obs.stride(1), scale,
                int(smooth), _lib.dtype_code(K.dtype), ws.data_ptr(), ws.numel(), _lib.stream_ptr(K.device))
    _lib.check(rc, "block_score")
    return out


def topk_blocks(scores: torch.Tensor, k: int) -> torch.Tensor:
    """Indices (int32, ascending) of the k highest scores; ties -> lowest index.

    scores [n] -> [k]; scores [rows, n] -> [rows, k], one selection per row
    (the per-KV-head mode)."""
    rows = int(scores.shape[0]) if scores.dim() == 2 else 1
    n = int(scores.shape[-1]) if scores.dim() >= 1 else 0
    k = max(0, min(int(k), n))
    out = torch.empty((rows, k) if scores.dim() == 2 else (k,), dtype=torch.int32, device=scores.device)
    if k == 0 or rows == 0:
        return out
    lib = _lib.lib()  # raises page16_native_unavailable when the library is missing
    s = scores.contiguous().float()
    with torch.cuda.device(s.device):
        rc = lib.bpkv_topk_select_batched(s.data_ptr(), n, k, rows, out.data_ptr(), _lib.stream_ptr(s.device))
    _lib.check(rc, "topk_select")
    return out


class BlockAlignedSnapKV:
    """Three-part block-aligned KV compression (sink | top-k mid blocks | obs tail).

    Same parameters and outputs as core/compress.py:23-175:
      L_final = sink_len + k_blocks*16 + obs_len, k_blocks = max(1, floor(r*N))
      (ratio mode) or floor((budget - sink - obs)/16) clipped to [0, N]
      (fixed-budget mode); inputs of length <= budget are returned unchanged.
    """

    def __init__(self, block_size: int = 16, sink_len: int = 64, obs_len: int = 64, retain_ratio: float = 0.20,
                 retain_budget_tokens: int = 0, per_kv_head: bool = False):
        if int(block_size) != 16:
            raise RuntimeError(f"page16_native_shape_unsupported:block_size_{block_size}")
        self.B = int(block_size)
        self.Ls = int(sink_len)
        self.Lo = int(obs_len)
        self.retain_ratio = retain_ratio
        self.retain_budget_tokens = max(0, int(retain_budget_tokens))
        # per_kv_head (this build's addition): every KV head keeps its own top-k
        # blocks; retained_block_idx then holds one list per KV head per batch row
        self.per_kv_head = bool(per_kv_head)
        self.last_debug: Dict[str, Any] = {}

    @property
    def compression_mode(self) -> str:
        return "fixed_budget" if int(self.retain_budget_tokens) > 0 else "ratio"

    def _k_blocks(self, N: int) -> Tuple[int, str]:
        budget = int(self.retain_budget_tokens)
        if budget > 0:
            mid_budget_tokens = max(0, budget - self.Ls - self.Lo)
            return max(0, min(int(N), int(math.floor(mid_budget_tokens / self.B)))), "fixed_budget"
        return max(1, int(math.floor(self.retain_ratio * N))), "ratio"

    def compress(self, K: torch.Tensor, V: torch.Tensor, Q_obs: torch.Tensor, n_rep: int = 1
                 ) -> Tuple[torch.Tensor, torch.Tensor]:
        b, h_kv, L, d = K.shape
        budget = int(self.retain_budget_tokens)
        if budget > 0 and L <= budget:
            self.last_debug = {
                "block_size": int(self.B), "sink_len": int(self.Ls), "obs_len": int(self.Lo),
                "retain_ratio": float(self.retain_ratio), "retain_budget_tokens": int(budget),
                "compression_mode": "fixed_budget", "logical_seq_len": int(L), "mid_tokens_before_align": 0,
                "mid_tokens_aligned": 0, "mid_block_count": 0, "retained_block_count": 0,
                "effective_retained_tokens": int(L), "retained_block_idx": [],
                "compression_skipped": "input_le_budget",
            }
            return K, V
        assert L >= self.Ls + self.Lo + self.B, f"sequence too short ({L}): needs at least {self.Ls + self.Lo + self.B}"
        if int(Q_obs.shape[1]) != h_kv * int(n_rep):
            raise RuntimeError("selected_writeback_bad_score_shape:gqa")
        L_premid = L - self.Ls - self.Lo
        N = math.ceil(L_premid / self.B)
        k_blocks, mode = self._k_blocks(N)
        k_blocks = min(k_blocks, N)
        eff = self.Ls + k_blocks * self.B + self.Lo
        K_out = torch.empty((b, h_kv, eff, d), dtype=K.dtype, device=K.device)
        V_out = torch.empty_like(K_out)
        idx_all = []
        n_pages = math.ceil(eff / self.B)
        dense_pages = torch.arange(n_pages, dtype=torch.int32, device=K.device)
        for i in range(b):
            scores = block_scores(K[i], Q_obs[i].to(K.dtype), self.Ls, self.Lo, d ** -0.5, SMOOTH_ALWAYS,
                                  per_kv_head=self.per_kv_head)
            sel = topk_blocks(scores, k_blocks)
            idx_all.append(sel)
            write_pages(K_out[i], V_out[i], K[i], V[i], dense_pages, sel, k_blocks, self.Ls, self.Lo, dense_out=True)
        self.last_debug = {
            "block_size": int(self.B), "sink_len": int(self.Ls), "obs_len": int(self.Lo),
            "retain_ratio": float(self.retain_ratio), "retain_budget_tokens": int(budget),
            "compression_mode": mode, "logical_seq_len": int(L), "mid_tokens_before_align": int(L_premid),
            "mid_tokens_aligned": int(N * self.B), "mid_block_count": int(N),
            "retained_block_count": int(k_blocks), "effective_retained_tokens": int(eff),
            "retained_block_idx": [t.long().cpu().tolist() for t in idx_all],
            "selection_scope": "per_kv_head" if self.per_kv_head else "shared",
        }
        return K_out, V_out
