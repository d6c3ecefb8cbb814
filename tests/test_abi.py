"""CPU tests of the C-ABI boundary: libbpkv.so loads here (no GPU needed) and
exports every entry point declared in include/bpkv.h; no compute is called."""
import ctypes
import re
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent


def _declared():
    text = (ROOT / "include" / "bpkv.h").read_text()
    return sorted(set(re.findall(r"BPKV_API\s+[\w\s\*]+?\b(bpkv_\w+)\s*\(", text)))


def test_header_declares_entry_points():
    names = _declared()
    assert "bpkv_page16_decode" in names and "bpkv_block_score" in names and len(names) >= 15


def test_library_exports_every_declared_symbol():
    from unifiedkv_b200 import _lib
    lib = ctypes.CDLL(str(_lib.LIB_PATH))
    missing = [n for n in _declared() if not hasattr(lib, n)]
    assert not missing, missing
    assert set(_declared()) <= set(_lib.SIGNATURES), "ctypes binding must cover the header"


def test_version_and_errors_without_gpu():
    from unifiedkv_b200 import _lib
    L = _lib.load()
    assert L.bpkv_version() >= 100
    # argument validation runs before any device work
    rc = L.bpkv_page16_decode(None, None, None, None, None, None, None, 2, 6, 4, 64, 1, 0, 0, 0, 0, 0.1, 2,
                              None, 0, None)
    assert rc == _lib.BPKV_ERR_SHAPE and "gqa" in _lib.last_error()
    rc = L.bpkv_topk_select(None, 10, 11, None, None)
    assert rc == _lib.BPKV_ERR_SHAPE


def test_new_entry_points_validate_without_gpu():
    """Argument checks of the per-KV-head, fused-append and peer-exchange entry points
    run before any device work."""
    from unifiedkv_b200 import _lib
    L = _lib.load()
    assert L.bpkv_peer_exchange_bytes(0, 32, 128) == 0 and L.bpkv_peer_exchange_bytes(9, 32, 128) == 0
    assert L.bpkv_peer_exchange_bytes(2, 32, 128) >= 2 * 2 * 32 * 132 * 4
    rc = L.bpkv_split_kv_merge_p2p(None, None, None, 3, 2, 32, 128, 100, None, None, None, 2, 2, None)
    assert rc == _lib.BPKV_ERR_SHAPE and "rank_3_of_2" in _lib.last_error()
    rc = L.bpkv_split_kv_merge_p2p(None, None, None, 0, 2, 32, 126, 100, None, None, None, 2, 2, None)
    assert rc == _lib.BPKV_ERR_SHAPE and "head_dim" in _lib.last_error()
    # fused split-KV decode: rank / head_dim / out dtype / peer buffers are checked first
    args = [None] * 7 + [1, 32, 8, 128, 10, 0, 0, 0, 0, 0.1, 2, 2, None, 0, 0]
    rc = L.bpkv_split_kv_decode_p2p(*args, None, 2, 2, 100, None, None)
    assert rc == _lib.BPKV_ERR_SHAPE and "rank_2_of_2" in _lib.last_error()
    dummy = ctypes.c_int(0)
    rc = L.bpkv_split_kv_decode_p2p(*args, None, 0, 2, 100, ctypes.byref(dummy), None)
    assert rc == _lib.BPKV_ERR_SHAPE and "null_pointer" in _lib.last_error()
    bad = list(args)
    bad[18] = 1  # out_dtype fp16 with bf16 inputs
    rc = L.bpkv_split_kv_decode_p2p(*bad, None, 0, 1, 100, ctypes.byref(dummy), None)
    assert rc == _lib.BPKV_ERR_SHAPE and "out_dtype" in _lib.last_error()
    rc = L.bpkv_split_kv_decode_p2p(*args, None, 0, 1, 100, ctypes.byref(dummy), None)
    assert rc == _lib.BPKV_ERR_SHAPE and "null_pointer" in _lib.last_error()  # q is NULL
    rc = L.bpkv_topk_select_batched(None, 10, 3, -1, None, None)
    assert rc == _lib.BPKV_ERR_SHAPE
    rc = L.bpkv_page_compact_per_kv_head(None, None, None, None, None, 3, 4, None, 100, 16, 16, 8, 128,
                                         0, 0, 0, 0, 0, 2, None)
    assert rc == _lib.BPKV_ERR_SHAPE and "selected_stride" in _lib.last_error()
    rc = L.bpkv_page16_decode_append(None, None, None, 0, None, None, None, None, None, None, 2, 8, 2, 64, 1,
                                     0, 0, 0, 0, 0.1, 2, None, 0, None)
    assert rc == _lib.BPKV_ERR_SHAPE and "null_new_token" in _lib.last_error()


def test_missing_library_fails_loudly():
    """No CPU fallback: with the library missing, the reference's flag reads False and
    every entry point raises (reference token page16_native_unavailable) instead of
    computing anything.  Run in a fresh interpreter so the real library is not cached."""
    import subprocess
    import sys
    from pathlib import Path
    code = r'''
import torch
from pathlib import Path
import unifiedkv_b200._lib as L
L.LIB_PATH = Path("/nonexistent/libbpkv.so")
from unifiedkv_b200 import page16_native, compress, chunked_prefill, pool, varlen
assert page16_native.HAS_TRITON is False and page16_native.HAS_PAGE16_NATIVE is False
calls = {
    "decode": lambda: page16_native.page16_decode_attention(
        torch.zeros(1, 4, 64), torch.zeros(2, 16, 1, 64), torch.zeros(2, 16, 1, 64),
        torch.zeros(1, 2, dtype=torch.int32), torch.ones(1, dtype=torch.int32), softmax_scale=0.125, n_rep=4),
    "scores": lambda: compress.block_scores(torch.zeros(1, 64, 64), torch.zeros(4, 8, 64), 8, 8),
    "topk": lambda: compress.topk_blocks(torch.zeros(10), 3),
    "append": lambda: page16_native.decode_append(
        torch.zeros(1, 1, 64), torch.zeros(1, 1, 64), torch.zeros(2, 16, 1, 64), torch.zeros(2, 16, 1, 64),
        torch.zeros(1, 2, dtype=torch.int32), torch.zeros(1, dtype=torch.int32)),
    "combine": lambda: page16_native.lse_combine(torch.zeros(2, 4, 64), torch.zeros(2, 4)),
    "writeback": lambda: pool.write_pages(torch.zeros(4, 16, 1, 64), torch.zeros(4, 16, 1, 64),
                                          torch.zeros(1, 64, 64), torch.zeros(1, 64, 64), [0, 1],
                                          torch.zeros(1, dtype=torch.int32), 1, 16, 16),
    "prefill": lambda: chunked_prefill.paged_chunk_prefill(
        torch.zeros(4, 4, 64), torch.zeros(2, 16, 1, 64), torch.zeros(2, 16, 1, 64),
        torch.zeros(1, 2, dtype=torch.int32), [0], [4], 0.125, 4),
}
for name, fn in calls.items():
    try:
        fn()
    except RuntimeError as exc:
        assert str(exc).startswith("page16_native_unavailable"), (name, str(exc))
    else:
        raise AssertionError(name + " ran without the library")
try:  # the reference's varlen entry raises ImportError without its backend (core/varlen.py:4-9)
    varlen.varlen_prefill_attention(torch.zeros(4, 4, 64), torch.zeros(4, 1, 64), torch.zeros(4, 1, 64), [4])
except ImportError:
    pass
else:
    raise AssertionError("varlen ran without the library")
assert varlen.HAS_FLASH_ATTN is False
print("ok")
'''
    root = Path(__file__).resolve().parents[1]
    r = subprocess.run([sys.executable, "-c", code], cwd=root, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and r.stdout.strip().endswith("ok"), r.stderr[-3000:]


def test_decode_shape_errors_in_reference_order():
    """Every shape check of page16_decode_attention raises the reference's token
    (core/page16_native.py:101-124), in the reference's order; the checks run
    before any device work, so CPU tensors reach them here."""
    import pytest
    import torch
    from unifiedkv_b200.page16_native import page16_decode_attention

    def call(q, k, v, bt, lens, n_rep=2):
        return page16_decode_attention(q, k, v, bt, lens, softmax_scale=0.1, n_rep=n_rep)

    q = torch.zeros(2, 4, 64)
    kc = torch.zeros(3, 16, 2, 64)
    bt = torch.zeros(2, 3, dtype=torch.int32)
    lens = torch.ones(2, dtype=torch.int32)
    cases = [
        (lambda: call(q[0], kc, kc, bt, lens), "q_dim_2"),
        (lambda: call(q, kc[0], kc, bt, lens), "cache_rank"),
        (lambda: call(q, kc[:, :8], kc[:, :8], bt, lens), "block_size_8"),
        (lambda: call(q, kc, kc, bt[0], lens), "block_table_rank"),
        (lambda: call(q[:0], kc, kc, bt[:0], lens[:0]), "empty"),
        (lambda: call(q, kc, kc[:, :, :1], bt, lens), "v_cache"),
        (lambda: call(torch.zeros(2, 3, 64), kc, kc, bt, lens), "gqa"),
        (lambda: call(q, kc, kc, bt[:1], lens), "block_table_batch"),
        (lambda: call(q, kc, kc, bt, lens[:1]), "seqlens"),
        (lambda: call(torch.zeros(2, 4, 512), torch.zeros(3, 16, 2, 512), torch.zeros(3, 16, 2, 512), bt, lens),
         "head_dim_512"),
        (lambda: call(q, kc, kc, bt, lens, n_rep=1), "gqa"),  # n_rep disagreeing with the head counts
    ]
    for fn, token in cases:
        with pytest.raises(RuntimeError, match=f"^page16_native_shape_unsupported:{token}$"):
            fn()
    # valid shapes on host tensors: refused before any launch
    with pytest.raises(RuntimeError, match="^page16_native_unavailable:tensors_not_on_cuda$"):
        call(q, kc, kc, bt, lens)
