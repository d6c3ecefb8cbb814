"""ctypes binding of libbpkv.so (declared in include/bpkv.h).

Every product entry point of this package goes through here.  There is no CPU
fallback: if the library is missing or cannot be loaded, calls raise
``RuntimeError("page16_native_unavailable:...")`` (the reference's token for a
missing native path, core/page16_native.py:100-101).
"""
from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

import torch

_PKG = Path(__file__).resolve().parent
LIB_PATH = _PKG / "lib" / ("libbpkv_trace.so" if os.environ.get("BPKV_TRACE") == "1" else "libbpkv.so")

BPKV_OK, BPKV_ERR_SHAPE, BPKV_ERR_UNSUPPORTED, BPKV_ERR_CUDA, BPKV_ERR_WORKSPACE = 0, 1, 2, 3, 4
BPKV_F32, BPKV_F16, BPKV_BF16 = 0, 1, 2

_DTYPE_CODE = {torch.float32: BPKV_F32, torch.float16: BPKV_F16, torch.bfloat16: BPKV_BF16}

_c_int, _c_i64, _c_sz, _c_f, _c_p = ctypes.c_int, ctypes.c_int64, ctypes.c_size_t, ctypes.c_float, ctypes.c_void_p
_c_u32 = ctypes.c_uint32

# name -> (restype, argtypes); must match include/bpkv.h
SIGNATURES = {
    "bpkv_last_error": (ctypes.c_char_p, []),
    "bpkv_version": (_c_int, []),
    "bpkv_build_hash": (ctypes.c_char_p, []),
    "bpkv_num_sms": (_c_int, []),
    "bpkv_debug_exp2_rate": (_c_int, [_c_int, _c_int, _c_p, _c_p]),
    "bpkv_debug_exp2_count": (ctypes.c_longlong, [_c_int, _c_int]),
    "bpkv_page16_decode_workspace_size": (_c_sz, [_c_int, _c_int, _c_int, _c_int, _c_int]),
    "bpkv_page16_decode": (_c_int, [_c_p, _c_p, _c_p, _c_p, _c_p, _c_p, _c_p,
                                    _c_int, _c_int, _c_int, _c_int, _c_int,
                                    _c_i64, _c_i64, _c_i64, _c_i64, _c_f, _c_int,
                                    _c_p, _c_sz, _c_p]),
    "bpkv_page16_decode_append": (_c_int, [_c_p, _c_p, _c_p, _c_i64, _c_p, _c_p, _c_p, _c_p, _c_p, _c_p,
                                           _c_int, _c_int, _c_int, _c_int, _c_int,
                                           _c_i64, _c_i64, _c_i64, _c_i64, _c_f, _c_int, _c_p, _c_sz, _c_p]),
    "bpkv_page16_decode_noalloc_max_scratch": (_c_sz, []),
    "bpkv_page16_decode_noalloc": (_c_int, [_c_p, _c_p, _c_p, _c_p, _c_p, _c_p, _c_p,
                                            _c_int, _c_int, _c_int, _c_int, _c_int,
                                            _c_i64, _c_i64, _c_i64, _c_i64, _c_f, _c_int, _c_p]),
    "bpkv_lse_combine": (_c_int, [_c_p, _c_p, _c_p, _c_p, _c_int, _c_int, _c_int, _c_int, _c_p]),
    "bpkv_peer_exchange_bytes": (_c_sz, [_c_int, _c_int, _c_int]),
    "bpkv_peer_buffer_alloc": (_c_int, [_c_sz, ctypes.POINTER(_c_p), _c_p]),
    "bpkv_peer_buffer_open": (_c_int, [_c_p, ctypes.POINTER(_c_p)]),
    "bpkv_peer_buffer_close": (_c_int, [_c_p]),
    "bpkv_peer_buffer_free": (_c_int, [_c_p]),
    "bpkv_split_kv_merge_p2p": (_c_int, [_c_p, _c_p, _c_p, _c_int, _c_int, _c_int, _c_int, _c_u32, _c_p, _c_p,
                                         _c_p, _c_int, _c_int, _c_p]),
    "bpkv_split_kv_decode_p2p": (_c_int, [_c_p, _c_p, _c_p, _c_p, _c_p, _c_p, _c_p,
                                          _c_int, _c_int, _c_int, _c_int, _c_int,
                                          _c_i64, _c_i64, _c_i64, _c_i64, _c_f, _c_int, _c_int,
                                          _c_p, _c_sz, _c_int, _c_p, _c_int, _c_int, _c_u32, _c_p, _c_p]),
    "bpkv_decode_append": (_c_int, [_c_p, _c_p, _c_p, _c_p, _c_p, _c_p, _c_int, _c_int, _c_int, _c_int,
                                    _c_i64, _c_i64, _c_i64, _c_int, _c_p]),
    "bpkv_block_score_workspace_size": (_c_sz, [_c_int, _c_int, _c_int, _c_int, _c_int]),
    "bpkv_block_score": (_c_int, [_c_p, _c_p, _c_p, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int,
                                  _c_i64, _c_i64, _c_i64, _c_i64, _c_f, _c_int, _c_int, _c_p, _c_sz, _c_p]),
    "bpkv_block_score_per_kv_head": (_c_int, [_c_p, _c_p, _c_p, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int,
                                              _c_int, _c_i64, _c_i64, _c_i64, _c_i64, _c_f, _c_int, _c_int, _c_p,
                                              _c_sz, _c_p]),
    "bpkv_topk_select": (_c_int, [_c_p, _c_int, _c_int, _c_p, _c_p]),
    "bpkv_topk_select_batched": (_c_int, [_c_p, _c_int, _c_int, _c_int, _c_p, _c_p]),
    "bpkv_page_compact_per_kv_head": (_c_int, [_c_p, _c_p, _c_p, _c_p, _c_p, _c_i64, _c_int, _c_p, _c_int, _c_int,
                                               _c_int, _c_int, _c_int, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64,
                                               _c_int, _c_p]),
    "bpkv_page_compact": (_c_int, [_c_p, _c_p, _c_p, _c_p, _c_p, _c_int, _c_p, _c_int, _c_int, _c_int,
                                   _c_int, _c_int, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_int, _c_p]),
    "bpkv_paged_prefill": (_c_int, [_c_p, _c_p, _c_p, _c_p, _c_p, _c_p, _c_p, _c_int, _c_int, _c_int,
                                    _c_int, _c_int, _c_int, _c_i64, _c_i64, _c_f, _c_int, _c_int, _c_p]),
    "bpkv_varlen_prefill": (_c_int, [_c_p, _c_p, _c_p, _c_p, _c_p, _c_int, _c_int, _c_int, _c_int, _c_int,
                                     _c_f, _c_int, _c_int, _c_p]),
    "bpkv_page_gather": (_c_int, [_c_p, _c_p, _c_int, _c_p, _c_i64, _c_i64, _c_int, _c_p]),
    "bpkv_page_scatter": (_c_int, [_c_p, _c_p, _c_int, _c_p, _c_i64, _c_i64, _c_int, _c_p]),
}

_lock = threading.Lock()
_lib = None
_load_error = None


def load(path: os.PathLike | None = None) -> ctypes.CDLL:
    """Load libbpkv.so (once) and bind every declared symbol."""
    global _lib, _load_error
    with _lock:
        if _lib is not None:
            return _lib
        p = Path(path) if path else LIB_PATH
        try:
            lib = ctypes.CDLL(str(p))
        except OSError as exc:  # missing or unloadable library: no fallback
            _load_error = f"{p}: {exc}"
            raise RuntimeError(f"page16_native_unavailable:lib_not_loaded:{_load_error}") from exc
        missing = []
        for name, (res, args) in SIGNATURES.items():
            try:
                fn = getattr(lib, name)
            except AttributeError:
                missing.append(name)
                continue
            fn.restype = res
            fn.argtypes = args
        if missing:  # a library built from other sources: refuse it now, not at the first call
            _load_error = f"{p}: missing symbols {missing}"
            raise RuntimeError(f"page16_native_unavailable:stale_library:missing_{','.join(missing)}")
        _check_build_hash(lib, p)
        _lib = lib
        return lib


def _check_build_hash(lib: ctypes.CDLL, p: Path) -> None:
    """The library must have been built from the sources beside it (when they are
    present: the package tree always ships them)."""
    global _load_error
    from . import build as _build
    if not _build.CSRC.is_dir() or not any(_build.CSRC.glob("*.cu")):
        return
    want = _build.tree_hash()
    have = lib.bpkv_build_hash().decode("ascii", "replace")
    if have != want:
        _load_error = f"{p}: built from sources {have}, tree is {want}"
        raise RuntimeError(f"page16_native_unavailable:stale_library:built_{have}_tree_{want}"
                           " (rebuild with python -m unifiedkv_b200.build)")


def available() -> bool:
    try:
        load()
        return True
    except RuntimeError:
        return False


def lib() -> ctypes.CDLL:
    return _lib if _lib is not None else load()


def last_error() -> str:
    return lib().bpkv_last_error().decode("utf-8", "replace")


def check(rc: int, what: str) -> None:
    """Map a non-zero return code to the reference-style RuntimeError."""
    if rc == BPKV_OK:
        return
    msg = last_error() or f"{what}_failed_rc_{rc}"
    if rc == BPKV_ERR_CUDA:
        raise RuntimeError(f"{msg}")
    raise RuntimeError(msg)


def dtype_code(dt: torch.dtype) -> int:
    try:
        return _DTYPE_CODE[dt]
    except KeyError:
        raise RuntimeError(f"page16_native_shape_unsupported:dtype_{dt}") from None


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream_ptr(device: torch.device | None = None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


_ws_cache: dict = {}


def workspace_for(nbytes: int, device: torch.device, stream, tag: str) -> torch.Tensor:
    """Like ``workspace`` for a stream object the caller already holds.  The
    library calls run with that stream current on the tensor's device (the
    caller's device context), so no device switch is needed here."""
    key = (device.index, stream.cuda_stream, tag)
    buf = _ws_cache.get(key)
    if buf is None or buf.numel() < nbytes:
        with torch.cuda.device(device):
            buf = torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=device)
        _ws_cache[key] = buf
    return buf


def workspace(nbytes: int, device: torch.device, tag: str = "default") -> torch.Tensor:
    """A per-(device, stream, tag) byte buffer reused across calls.

    Calls on one stream are ordered, so reusing one buffer per stream is safe;
    it only grows.
    """
    st = torch.cuda.current_stream(device).cuda_stream
    key = (device.index if device.index is not None else torch.cuda.current_device(), st, tag)
    buf = _ws_cache.get(key)
    if buf is None or buf.numel() < nbytes:
        buf = torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=device)
        _ws_cache[key] = buf
    return buf
