"""Page16 decode oracle (numpy).  TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).

Restates the reference's PyTorch gather-then-attention path:
  * page gather and trim to each request's length: core/engine.py:4060-4100
    (index_select pages -> [B, h_kv, max_blocks*16, d] -> slice to len);
  * GQA expansion: repeat_kv, core/compress.py:7-20;
  * attention: softmax(scale * q . K^T) . V, with the same length semantics as
    the Triton kernel core/page16_native.py:53-73 (pages past ``max_blocks``
    are never read; a request with no valid token gives 0/0 = NaN).
"""
from __future__ import annotations

import numpy as np


def gather_request_kv(k_cache, v_cache, block_table_row, length):
    """K, V of one request as [h_kv, T, d] (engine.py:4060-4100 restated)."""
    max_blocks = block_table_row.shape[0]
    n = min(int(length), 16 * max_blocks)
    if n <= 0:
        shape = (k_cache.shape[2], 0, k_cache.shape[3])
        return np.zeros(shape, k_cache.dtype), np.zeros(shape, v_cache.dtype)
    npages = (n + 15) // 16
    ids = block_table_row[:npages].astype(np.int64)
    k = k_cache[ids].reshape(npages * 16, k_cache.shape[2], k_cache.shape[3])[:n]
    v = v_cache[ids].reshape(npages * 16, v_cache.shape[2], v_cache.shape[3])[:n]
    return np.ascontiguousarray(k.transpose(1, 0, 2)), np.ascontiguousarray(v.transpose(1, 0, 2))


def page16_decode_reference(q, k_cache, v_cache, block_table, cache_seqlens, softmax_scale, n_rep,
                            compute_dtype=np.float64, return_lse=False):
    """out[b, h] = softmax(scale * q[b,h] . K_b[h // n_rep]^T) . V_b[h // n_rep].

    q: [B, h_q, d]; k/v_cache: [N, 16, h_kv, d]; block_table: [B, max_blocks];
    cache_seqlens: [B].  Returns out [B, h_q, d] (compute_dtype) and, with
    return_lse, the natural-log sum-exp of the scaled logits [B, h_q].
    """
    q = np.asarray(q)
    B, hq, d = q.shape
    out = np.empty((B, hq, d), compute_dtype)
    lse = np.empty((B, hq), compute_dtype)
    for b in range(B):
        k, v = gather_request_kv(k_cache, v_cache, np.asarray(block_table[b]), int(cache_seqlens[b]))
        if k.shape[1] == 0:
            out[b] = np.nan
            lse[b] = -np.inf
            continue
        k = k.astype(compute_dtype, copy=False)
        v = v.astype(compute_dtype, copy=False)
        qb = q[b].astype(compute_dtype).reshape(k.shape[0], n_rep, -1)
        # repeat_kv semantics (q-head h reads kv-head h // n_rep), one BLAS matmul per kv head
        s = np.matmul(qb, k.transpose(0, 2, 1)).reshape(k.shape[0] * n_rep, -1) * compute_dtype(softmax_scale)
        m = s.max(axis=1, keepdims=True)
        p = np.exp(s - m)
        l = p.sum(axis=1, keepdims=True)
        pv = np.matmul(p.reshape(k.shape[0], n_rep, -1), v).reshape(k.shape[0] * n_rep, -1)
        out[b] = pv / l
        lse[b] = (m + np.log(l))[:, 0]
    return (out, lse) if return_lse else out


def lse_merge_reference(part_out, part_lse):
    """Merge split partials: part_out [P, rows, d], part_lse [P, rows] -> (out, lse)."""
    part_out = np.asarray(part_out, np.float64)
    part_lse = np.asarray(part_lse, np.float64)
    M = part_lse.max(axis=0)
    with np.errstate(invalid="ignore"):
        w = np.exp(part_lse - M[None])
    W = w.sum(axis=0)
    out = (w[..., None] * part_out).sum(axis=0) / W[:, None]
    return out, M + np.log(W)
