"""Compression / selection / writeback oracle (numpy).  TEST INFRASTRUCTURE ONLY
(see oracle/__init__.py).

Restates:
  * block scoring: core/compress.py:100-130 and core/scheduler.py:565-592
    (zero-padded K_mid, softmax over all padded tokens, mean over window
    queries, max over q-heads, 16-token block sums, max_pool1d(3, 1, 1));
  * top-k budget rules: core/compress.py:133-139 (compress) and
    core/scheduler.py:547-564 (selected writeback);
  * top-k: torch.topk + ascending sort (core/compress.py:141-142,
    core/scheduler.py:615-616) with the tie order fixed to lowest index first;
  * writeback source order: core/scheduler.py:666-799 (sink, selected mid blocks
    padded to 16, observation tail; slots past effective_len untouched).
Per-KV-head mode (no reference counterpart; the reference's selection is shared
across KV heads): the same score with the max taken only over the q heads of
one KV group, then the same top-k and writeback rules applied per KV head.
"""
from __future__ import annotations

import math

import numpy as np


def selection_budget_blocks(L, sink, obs, budget=0, ratio=0.2, B=16):
    """(k_blocks, effective_len, mode) as KVScheduler._selection_budget_blocks."""
    if budget > 0 and L <= budget:
        return 0, int(L), "input_le_budget"
    if L < sink + obs + B:
        return 0, int(L), "too_short"
    mid_tokens = max(0, L - sink - obs)
    mid_blocks = int(math.ceil(mid_tokens / B))
    if budget > 0:
        mid_budget = max(0, budget - sink - obs)
        k = max(0, min(mid_blocks, int(math.floor(mid_budget / B))))
        return k, sink + k * B + obs, "fixed_budget"
    k = max(1, min(mid_blocks, int(math.floor(float(ratio) * mid_blocks))))
    return k, sink + k * B + obs, "ratio"


def compress_k_blocks(N, sink, obs, budget=0, ratio=0.2, B=16):
    """k_blocks of BlockAlignedSnapKV.compress (core/compress.py:133-139)."""
    if budget > 0:
        mid_budget_tokens = max(0, budget - sink - obs)
        return max(0, min(int(N), int(math.floor(mid_budget_tokens / B))))
    return max(1, int(math.floor(ratio * N)))


def block_scores(K, Q, sink, obs, scale=None, smooth="always", dtype=np.float64, per_kv_head=False):
    """K [h_kv, L, d], Q [h_q, W, d] -> block scores [N] (dtype), or [h_kv, N] per KV head."""
    K = np.asarray(K, dtype)
    Q = np.asarray(Q, dtype)
    h_kv, L, d = K.shape
    h_q, W, _ = Q.shape
    n_rep = h_q // h_kv
    scale = d ** -0.5 if scale is None else scale
    mid = K[:, sink:L - obs, :]
    Lm = mid.shape[1]
    N = int(math.ceil(Lm / 16))
    if N <= 0:
        return np.zeros(0, dtype)
    pad = np.zeros((h_kv, N * 16, d), dtype)
    pad[:, :Lm] = mid
    S = np.full((h_kv, N * 16), -np.inf, dtype)  # per KV group: max over its q heads
    for hq in range(h_q):
        s = Q[hq] @ pad[hq // n_rep].T * dtype(scale)  # [W, T]
        s = s - s.max(axis=1, keepdims=True)
        p = np.exp(s)
        p /= p.sum(axis=1, keepdims=True)
        S[hq // n_rep] = np.maximum(S[hq // n_rep], p.mean(axis=0))
    if not per_kv_head:
        S = S.max(axis=0, keepdims=True)
    blk = S.reshape(S.shape[0], N, 16).sum(axis=2)
    if smooth == "always" or (smooth == "if3" and N >= 3):
        padded = np.concatenate([np.full((blk.shape[0], 1), -np.inf), blk, np.full((blk.shape[0], 1), -np.inf)], 1)
        blk = np.maximum(np.maximum(padded[:, :-2], padded[:, 1:-1]), padded[:, 2:])
    return blk if per_kv_head else blk[0]


def topk_lowest_index(scores, k):
    """Ascending indices of the k largest scores, ties broken by lowest index."""
    scores = np.asarray(scores)
    k = max(0, min(int(k), scores.shape[0]))
    order = np.lexsort((np.arange(scores.shape[0]), -scores))
    return np.sort(order[:k]).astype(np.int64)


def selection_is_consistent(selected, scores64, k, rel_tol=1e-5):
    """True if ``selected`` is a valid top-k of ``scores64`` up to near-ties.

    Blocks whose fp64 score lies within rel_tol of the k-th score may swap
    (different float reduction orders can flip them); everything strictly above
    that band must be selected and nothing strictly below it may be.
    """
    ref = topk_lowest_index(scores64, k)
    if k == 0:
        return len(selected) == 0
    kth = np.sort(scores64)[::-1][k - 1]
    band = rel_tol * max(abs(kth), 1e-30)
    sel = set(int(x) for x in selected)
    must = {i for i in range(len(scores64)) if scores64[i] > kth + band}
    never = {i for i in range(len(scores64)) if scores64[i] < kth - band}
    return len(sel) == len(ref) and must <= sel and not (sel & never)


def writeback_source_tokens(L, sink, obs, selected, uncompressed=False):
    """Source token (or -1 for zero padding) of every destination token."""
    if uncompressed:
        return np.arange(L, dtype=np.int64)
    k = len(selected)
    src = []
    src.extend(range(sink))
    mid_end = L - obs
    for idx in selected:
        for o in range(16):
            t = sink + 16 * int(idx) + o
            src.append(t if t < mid_end else -1)
    src.extend(range(L - obs, L))
    assert len(src) == sink + 16 * k + obs
    return np.asarray(src, np.int64)


def writeback_pool(k_pool, v_pool, K, V, dst_pages, src_tokens):
    """Apply a compacting writeback to copies of pool layers [N, 16, h, d].

    src_tokens: [eff] shared by all KV heads, or [h_kv, eff] per KV head."""
    kp, vp = k_pool.copy(), v_pool.copy()
    src = np.asarray(src_tokens)
    if src.ndim == 1:
        src = np.broadcast_to(src, (K.shape[0], src.shape[0]))
    for h in range(K.shape[0]):
        for p, t in enumerate(src[h]):
            page, slot = dst_pages[p // 16], p % 16
            if t < 0:
                kp[page, slot, h] = 0
                vp[page, slot, h] = 0
            else:
                kp[page, slot, h] = K[h, t, :]
                vp[page, slot, h] = V[h, t, :]
    return kp, vp


def compress(K, V, Q, sink, obs, budget=0, ratio=0.2):
    """BlockAlignedSnapKV.compress for one batch row: (K_final, V_final, selected) or None if skipped."""
    h_kv, L, d = K.shape
    if budget > 0 and L <= budget:
        return K, V, None
    N = int(math.ceil((L - sink - obs) / 16))
    k = compress_k_blocks(N, sink, obs, budget, ratio)
    scores = block_scores(K, Q, sink, obs)
    sel = topk_lowest_index(scores, k)
    src = writeback_source_tokens(L, sink, obs, sel)
    Kf = np.where(src[None, :, None] >= 0, K[:, np.maximum(src, 0), :], 0)
    Vf = np.where(src[None, :, None] >= 0, V[:, np.maximum(src, 0), :], 0)
    return Kf, Vf, sel


def compress_per_kv_head(K, V, Q, sink, obs, budget=0, ratio=0.2):
    """Per-KV-head variant of compress: (K_final, V_final, selected [h_kv][k]) or (K, V, None) if skipped."""
    h_kv, L, d = K.shape
    if budget > 0 and L <= budget:
        return K, V, None
    N = int(math.ceil((L - sink - obs) / 16))
    k = compress_k_blocks(N, sink, obs, budget, ratio)
    scores = block_scores(K, Q, sink, obs, per_kv_head=True)
    sels = [topk_lowest_index(scores[h], k) for h in range(h_kv)]
    Kf = np.zeros((h_kv, sink + 16 * k + obs, d), K.dtype)
    Vf = np.zeros_like(Kf)
    for h in range(h_kv):
        src = writeback_source_tokens(L, sink, obs, sels[h])
        Kf[h] = np.where(src[:, None] >= 0, K[h, np.maximum(src, 0), :], 0)
        Vf[h] = np.where(src[:, None] >= 0, V[h, np.maximum(src, 0), :], 0)
    return Kf, Vf, np.stack(sels) if k > 0 else np.zeros((h_kv, 0), np.int64)
