"""Causal chunked-prefill oracle (numpy).  TEST INFRASTRUCTURE ONLY.

The reference has no paged chunked-prefill attention: its chunks run through HF
flash_attention_2 over a dense cache (core/engine.py:304-305, :1772-1854).  The GPU
tests pin this restatement to that arithmetic (flash_attn_func on the dense K/V
gathered from the pages agrees with it within flash-attn's own bf16 error).  This
restates causal softmax attention with past context, bottom-right aligned as
flash-attn defines it for seqlen_q <= seqlen_k (query i of an n_q-token chunk
sees kv tokens t <= seqlen_k - n_q + i), which is also what
flash_attn_varlen_func(causal=True) computes for core/varlen.py:29-41 when
there is no past.
"""
from __future__ import annotations

import numpy as np


def chunk_attention(q, k, v, causal=True, scale=None, dtype=np.float64):
    """q [n_q, h_q, d]; k, v [n_k, h_kv, d] (past + chunk) -> [n_q, h_q, d]."""
    q = np.asarray(q, dtype)
    k = np.asarray(k, dtype)
    v = np.asarray(v, dtype)
    n_q, h_q, d = q.shape
    n_k, h_kv, _ = k.shape
    rep = h_q // h_kv
    scale = d ** -0.5 if scale is None else scale
    out = np.zeros((n_q, h_q, d), dtype)
    for h in range(h_q):
        s = q[:, h] @ k[:, h // rep].T * scale
        if causal:
            lim = n_k - n_q + np.arange(n_q)
            s = np.where(np.arange(n_k)[None, :] <= lim[:, None], s, -np.inf)
        m = s.max(axis=1, keepdims=True)
        ok = np.isfinite(m)[:, 0]
        p = np.exp(s - np.where(np.isfinite(m), m, 0))
        l = p.sum(axis=1, keepdims=True)
        out[ok, h] = (p @ v[:, h // rep])[ok] / l[ok]
    return out
