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
(run on CPU); see ``tests/golden/make_golden.py``.  The paged chunked-prefill
restatement has no reference implementation to pin it (the reference never
attends chunks over paged KV): parity unpinned for that part.
"""
