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
    rc = L.bpkv_split_kv_merge_p2p(None, None, None, 3, 2, 32, 128, 100, None, None, None, 2, None)
    assert rc == _lib.BPKV_ERR_SHAPE and "rank_3_of_2" in _lib.last_error()
    rc = L.bpkv_split_kv_merge_p2p(None, None, None, 0, 2, 32, 126, 100, None, None, None, 2, None)
    assert rc == _lib.BPKV_ERR_SHAPE and "head_dim" in _lib.last_error()
    rc = L.bpkv_topk_select_batched(None, 10, 3, -1, None, None)
    assert rc == _lib.BPKV_ERR_SHAPE
    rc = L.bpkv_page_compact_per_kv_head(None, None, None, None, None, 3, 4, None, 100, 16, 16, 8, 128,
                                         0, 0, 0, 0, 0, 2, None)
    assert rc == _lib.BPKV_ERR_SHAPE and "selected_stride" in _lib.last_error()
    rc = L.bpkv_page16_decode_append(None, None, None, 0, None, None, None, None, None, None, 2, 8, 2, 64, 1,
                                     0, 0, 0, 0, 0.1, 2, None, 0, None)
    assert rc == _lib.BPKV_ERR_SHAPE and "null_new_token" in _lib.last_error()
