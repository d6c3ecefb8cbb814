"""B200-native (sm_100a) hot path of the BP-KV block-paged KV runtime.

Drop-in modules mirroring the reference (majic-mk/UnifiedKV ``core/``):
  page16_native  - Page16 split-KV decode (core/page16_native.py)
  compress       - BlockAlignedSnapKV with fused GPU scoring (core/compress.py)
  selection      - selected-writeback scheduler methods (core/scheduler.py:547-878)
  pool, kv_types - paged pool and its metadata (core/pool.py, core/kv_types.py)
  varlen, chunked_prefill - prefill attention (core/varlen.py, core/chunked_prefill.py)
  multi_gpu      - request sharding and split-KV over NCCL (core/multi_gpu.py)
All compute runs in libbpkv.so (include/bpkv.h); there is no CPU fallback.
"""
from . import _lib  # noqa: F401

__all__ = ["_lib"]
__version__ = "0.1.0"
