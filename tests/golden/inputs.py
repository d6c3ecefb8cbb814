"""Seeded synthetic inputs shared by the golden-vector generator and the tests.

numpy's PCG64 ``default_rng`` stream is stable across numpy releases, so the
fixtures only store outputs plus a checksum of the inputs they were made from.
"""
from __future__ import annotations

import hashlib

import numpy as np


def checksum(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        a = np.ascontiguousarray(a)
        h.update(str(a.dtype).encode())
        h.update(str(a.shape).encode())
        h.update(a.tobytes())
    return h.hexdigest()[:16]


def page16_case(seed, batch, hq, hkv, d, lens, num_pages, max_blocks=None, dtype=np.float32, scale_std=1.0):
    """q [B,hq,d], k/v cache [N,16,hkv,d], block_table [B,max_blocks] int32, lens int32.

    Pages are drawn without replacement from a random permutation of the pool
    (core/pool.py keeps pages anywhere in the pool); unused table slots are
    0-padded as core/pool.py:174-189 does.
    """
    rng = np.random.default_rng(seed)
    lens = np.asarray(lens, np.int32)
    need = [(int(l) + 15) // 16 for l in lens]
    mb = max_blocks if max_blocks is not None else max(max(need), 1)
    assert sum(need) <= num_pages
    perm = rng.permutation(num_pages).astype(np.int32)
    bt = np.zeros((batch, mb), np.int32)
    off = 0
    for b, n in enumerate(need):
        n_use = min(n, mb)
        bt[b, :n_use] = perm[off:off + n_use]
        off += n
    q = (rng.standard_normal((batch, hq, d)) * scale_std).astype(dtype)
    k = (rng.standard_normal((num_pages, 16, hkv, d)) * scale_std).astype(dtype)
    v = (rng.standard_normal((num_pages, 16, hkv, d)) * scale_std).astype(dtype)
    return q, k, v, bt, lens


# Config 1 of the benchmark plan: B=2, 8/2 heads, d=64, lens (1000, 777), 256-page pool, fp32.
CONFIG1 = dict(seed=0, batch=2, hq=8, hkv=2, d=64, lens=(1000, 777), num_pages=256)

PAGE16_CASES = {
    "config1_fp32": CONFIG1,
    "gqa4_d128_fp16": dict(seed=1, batch=3, hq=8, hkv=2, d=128, lens=(37, 300, 16), num_pages=64,
                           max_blocks=24, dtype=np.float16),
    "mha_d64_len_cap": dict(seed=2, batch=2, hq=4, hkv=4, d=64, lens=(250, 100), num_pages=40,
                            max_blocks=10),  # request 0 longer than its table: pages past max_blocks unread
    "gqa8_d32_tiny": dict(seed=3, batch=4, hq=8, hkv=1, d=32, lens=(1, 15, 17, 33), num_pages=16),
}


def compress_case(seed, h_kv, L, d, n_rep, window, hot_blocks=0, sink=0, bias=2.0, dtype=np.float32):
    """K, V [h_kv, L, d] and Q_obs [h_kv*n_rep, window, d]; optional hot blocks whose keys
    are pulled toward the window queries by ``bias`` standard deviations."""
    rng = np.random.default_rng(seed)
    K = rng.standard_normal((h_kv, L, d)).astype(np.float64)
    V = rng.standard_normal((h_kv, L, d)).astype(np.float64)
    Q = rng.standard_normal((h_kv * n_rep, window, d)).astype(np.float64)
    hot = np.zeros(0, np.int64)
    if hot_blocks:
        n_blocks = L // 16
        hot = np.sort(rng.choice(np.arange(sink // 16, n_blocks), size=hot_blocks, replace=False))
        qdir = Q.reshape(h_kv, n_rep, window, d).mean(axis=(1, 2))
        qdir /= np.linalg.norm(qdir, axis=-1, keepdims=True)
        for blk in hot:
            # shift of per-coordinate RMS ``bias`` sigma along the mean query direction
            K[:, blk * 16:(blk + 1) * 16, :] += bias * np.sqrt(d) * qdir[:, None, :]
    return K.astype(dtype), V.astype(dtype), Q.astype(dtype), hot
