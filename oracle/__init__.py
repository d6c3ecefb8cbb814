"""CPU oracle for the BP-KV hot path — TEST INFRASTRUCTURE ONLY.

This package restates the reference algorithms (majic-mk/UnifiedKV, ``core/``)
in numpy so that the CUDA path can be checked against them.  Only ``tests/``,
``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl reference``
legs of ``bench.py`` may import it, and only as the checker or as the timed CPU
baseline; the product (``unifiedkv_b200``) never imports it and has no CPU
fallback.

Pinning: the decode restatement is checked against golden vectors produced by
the reference's own Triton kernel (run under TRITON_INTERPRET=1), and the
compression restatement against the reference's own ``BlockAlignedSnapKV``
(run on CPU, also once per KV head for the per-KV-head mode); see
``tests/golden/make_golden.py``.  The reference never attends chunks over paged
KV; its chunk path runs HF ``flash_attention_2`` over a dense cache, so the
chunked-prefill restatement is pinned on the GPU box instead: the tests compare
``flash_attn_func`` on the K/V gathered from the pages with this restatement
(and the build's kernel against both).
"""
