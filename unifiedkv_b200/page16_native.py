"""Drop-in replacement for the reference module ``page16_native``.

Reference: core/page16_native.py:83-150 (``page16_decode_attention``) and the
import site core/scheduler.py:13-17, which reads
``from page16_native import HAS_TRITON as HAS_PAGE16_NATIVE, page16_decode_attention``.
The name ``HAS_TRITON`` is kept for that import; here it means "the native
sm_100a library (libbpkv.so) is loaded".  There is no Triton and no CPU
fallback: when the library is absent the call raises the reference's
``page16_native_unavailable`` error.
"""
from __future__ import annotations

import torch

from . import _lib

HAS_TRITON = _lib.available()
HAS_PAGE16_NATIVE = HAS_TRITON


def _check_shapes(q, k_cache, v_cache, block_table, cache_seqlens):
    """Argument validation with the reference's exact error tokens
    (core/page16_native.py:100-124)."""
    if not HAS_TRITON:
        raise RuntimeError("page16_native_unavailable:native_library_not_loaded")
    if q.dim() != 3:
        raise RuntimeError(f"page16_native_shape_unsupported:q_dim_{q.dim()}")
    if k_cache.dim() != 4 or v_cache.dim() != 4:
        raise RuntimeError("page16_native_shape_unsupported:cache_rank")
    if int(k_cache.shape[1]) != 16:
        raise RuntimeError(f"page16_native_shape_unsupported:block_size_{int(k_cache.shape[1])}")
    if block_table.dim() != 2:
        raise RuntimeError("page16_native_shape_unsupported:block_table_rank")
    batch, num_q_heads, head_dim = [int(x) for x in q.shape]
    num_kv_heads = int(k_cache.shape[2])
    if batch <= 0 or num_q_heads <= 0 or head_dim <= 0:
        raise RuntimeError("page16_native_shape_unsupported:empty")
    if int(v_cache.shape[1]) != 16 or int(v_cache.shape[2]) != num_kv_heads or int(v_cache.shape[3]) != head_dim:
        raise RuntimeError("page16_native_shape_unsupported:v_cache")
    if num_q_heads % num_kv_heads != 0:
        raise RuntimeError("page16_native_shape_unsupported:gqa")
    if int(block_table.shape[0]) != batch:
        raise RuntimeError("page16_native_shape_unsupported:block_table_batch")
    if int(cache_seqlens.numel()) != batch:
        raise RuntimeError("page16_native_shape_unsupported:seqlens")
    if head_dim > 256:
        raise RuntimeError(f"page16_native_shape_unsupported:head_dim_{head_dim}")
    return batch, num_q_heads, num_kv_heads, head_dim


def _page_view_ok(cache: torch.Tensor, num_kv_heads: int, head_dim: int) -> bool:
    """The kernel needs each page's [16, h_kv, d] block dense (any page stride)."""
    s = cache.stride()
    return s[3] == 1 and s[2] == head_dim and s[1] == num_kv_heads * head_dim


def _prepare(q, k_cache, v_cache, block_table, cache_seqlens, n_rep):
    """Shared validation of the decode entry points (the reference's checks and
    tokens, core/page16_native.py:100-128): returns q, block_table and
    cache_seqlens made contiguous int32 / contiguous, and the four sizes."""
    batch, num_q_heads, num_kv_heads, head_dim = _check_shapes(q, k_cache, v_cache, block_table, cache_seqlens)
    if int(n_rep) != num_q_heads // num_kv_heads:
        raise RuntimeError("page16_native_shape_unsupported:gqa")
    if not (q.is_cuda and k_cache.is_cuda and v_cache.is_cuda and block_table.is_cuda and cache_seqlens.is_cuda):
        raise RuntimeError("page16_native_unavailable:tensors_not_on_cuda")
    if k_cache.dtype != q.dtype or v_cache.dtype != q.dtype:
        raise RuntimeError("page16_native_shape_unsupported:dtype_mismatch")
    if not _page_view_ok(k_cache, num_kv_heads, head_dim) or not _page_view_ok(v_cache, num_kv_heads, head_dim):
        raise RuntimeError("page16_native_shape_unsupported:cache_layout")
    if k_cache.stride(0) != v_cache.stride(0):
        raise RuntimeError("page16_native_shape_unsupported:cache_layout")
    q = q.contiguous()
    if block_table.dtype != torch.int32:
        block_table = block_table.to(torch.int32)
    block_table = block_table.contiguous()
    cache_seqlens = cache_seqlens.to(dtype=torch.int32).contiguous()
    return q, block_table, cache_seqlens, (batch, num_q_heads, num_kv_heads, head_dim)


def page16_decode_attention(
    q: torch.Tensor,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    block_table: torch.Tensor,
    cache_seqlens: torch.Tensor,
    *,
    softmax_scale: float,
    n_rep: int,
    lse_out: torch.Tensor | None = None,
    k_new: torch.Tensor | None = None,
    v_new: torch.Tensor | None = None,
) -> torch.Tensor:
    """Decode-only paged attention over 16-token pages (sm_100a split-KV kernel).

    Same contract as the reference (core/page16_native.py:83-150):
      q: [batch, num_q_heads, head_dim] CUDA tensor (made contiguous here).
      k_cache/v_cache: [num_blocks, 16, num_kv_heads, head_dim] (one layer's view).
      block_table: [batch, max_blocks] int32 (0-padded).
      cache_seqlens: [batch] lengths including the current token (cast to int32).
    Returns ``empty_like(q)`` filled with the attention output, computed on the
    current stream without synchronising.  ``n_rep`` is implied by the head
    counts (as in the reference kernel, where kv_h = q_head // n_rep); a value
    that disagrees is rejected with the ``gqa`` token.

    ``lse_out`` (optional, this build's addition): fp32 [batch, num_q_heads]
    receives the natural-log sum-exp of the scaled logits, used to merge
    split-KV partials across GPUs.

    ``k_new``/``v_new`` (optional, this build's addition): [batch, num_kv_heads,
    head_dim] rows of this step's token.  The launch stores them into the pool
    at position ``cache_seqlens[b] - 1`` and attends over them in the same pass,
    replacing the scatter-then-attend pair of direct_forward
    (core/scheduler.py:398-418).
    """
    q, block_table, cache_seqlens, (batch, num_q_heads, num_kv_heads, head_dim) = _prepare(
        q, k_cache, v_cache, block_table, cache_seqlens, n_rep)
    out = torch.empty_like(q)
    if lse_out is not None:
        if lse_out.dtype != torch.float32 or lse_out.numel() != batch * num_q_heads or not lse_out.is_contiguous():
            raise RuntimeError("page16_native_shape_unsupported:lse_out")
    if (k_new is None) != (v_new is None):
        raise RuntimeError("page16_native_shape_unsupported:new_token")
    if k_new is not None:
        want = (batch, num_kv_heads, head_dim)
        if tuple(k_new.shape) != want or tuple(v_new.shape) != want:
            raise RuntimeError("page16_native_shape_unsupported:new_token")
        if k_new.dtype != q.dtype or v_new.dtype != q.dtype or not (k_new.is_cuda and v_new.is_cuda):
            raise RuntimeError("page16_native_shape_unsupported:new_token")
        k_new = k_new.contiguous()
        v_new = v_new.contiguous()
    dev = q.device
    if dev.index != torch.cuda.current_device():  # the library launches on the current device
        with torch.cuda.device(dev):
            return page16_decode_attention(q, k_cache, v_cache, block_table, cache_seqlens,
                                           softmax_scale=softmax_scale, n_rep=n_rep, lse_out=lse_out,
                                           k_new=k_new, v_new=v_new)
    L = _lib.lib()
    code = _lib.dtype_code(q.dtype)
    stream = torch.cuda.current_stream(dev)
    ws = _lib.workspace_for(L.bpkv_page16_decode_workspace_size(batch, num_q_heads, num_kv_heads, head_dim, code),
                            dev, stream, "page16")
    if k_new is None:
        rc = L.bpkv_page16_decode(
            q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), block_table.data_ptr(),
            cache_seqlens.data_ptr(), out.data_ptr(), _lib.ptr(lse_out),
            batch, num_q_heads, num_kv_heads, head_dim, int(block_table.shape[1]),
            q.stride(0), q.stride(1), k_cache.stride(0), block_table.stride(0),
            float(softmax_scale), code, ws.data_ptr(), ws.numel(), stream.cuda_stream)
    else:
        rc = L.bpkv_page16_decode_append(
            q.data_ptr(), k_new.data_ptr(), v_new.data_ptr(), k_new.stride(0),
            k_cache.data_ptr(), v_cache.data_ptr(), block_table.data_ptr(),
            cache_seqlens.data_ptr(), out.data_ptr(), _lib.ptr(lse_out),
            batch, num_q_heads, num_kv_heads, head_dim, int(block_table.shape[1]),
            q.stride(0), q.stride(1), k_cache.stride(0), block_table.stride(0),
            float(softmax_scale), code, ws.data_ptr(), ws.numel(), stream.cuda_stream)
    _lib.check(rc, "page16_native")
    return out


def decode_append(k_new: torch.Tensor, v_new: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                  block_table: torch.Tensor, old_lens: torch.Tensor) -> None:
    """Write this step's k/v ([batch, h_kv, d]) at slot (block_table[b, old/16], old % 16).

    Device-side replacement of the indexed scatter in direct_forward
    (core/scheduler.py:398-408); no host synchronisation.
    """
    batch, h_kv, d = [int(x) for x in k_new.shape]
    if v_new.shape != k_new.shape or k_cache.shape[1] != 16 or k_cache.shape[2] != h_kv or k_cache.shape[3] != d:
        raise RuntimeError("decode_append_shape_unsupported:shape")
    if not (_page_view_ok(k_cache, h_kv, d) and _page_view_ok(v_cache, h_kv, d)) or k_cache.stride(0) != v_cache.stride(0):
        raise RuntimeError("decode_append_shape_unsupported:cache_layout")
    k_new = k_new.contiguous()
    v_new = v_new.contiguous()
    bt = block_table.to(torch.int32).contiguous()
    lens = old_lens.to(torch.int32).contiguous()
    dev = k_new.device
    lib = _lib.lib()  # raises page16_native_unavailable when the library is missing
    with torch.cuda.device(dev):
        rc = lib.bpkv_decode_append(
            k_new.data_ptr(), v_new.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), bt.data_ptr(),
            lens.data_ptr(), batch, h_kv, d, int(bt.shape[1]), k_new.stride(0), k_cache.stride(0), bt.stride(0),
            _lib.dtype_code(k_new.dtype), _lib.stream_ptr(dev))
    _lib.check(rc, "decode_append")


def lse_combine(part_out: torch.Tensor, part_lse: torch.Tensor, out_dtype: torch.dtype = torch.bfloat16,
                return_lse: bool = False):
    """Merge split-KV partials: part_out fp32 [P, rows, d], part_lse fp32 [P, rows]."""
    P, rows, d = [int(x) for x in part_out.shape]
    part_out = part_out.contiguous().float()
    part_lse = part_lse.contiguous().float()
    out = torch.empty(rows, d, dtype=out_dtype, device=part_out.device)
    lse = torch.empty(rows, dtype=torch.float32, device=part_out.device) if return_lse else None
    lib = _lib.lib()  # raises page16_native_unavailable when the library is missing
    with torch.cuda.device(part_out.device):
        rc = lib.bpkv_lse_combine(part_out.data_ptr(), part_lse.data_ptr(), out.data_ptr(), _lib.ptr(lse),
                                  P, rows, d, _lib.dtype_code(out_dtype), _lib.stream_ptr(part_out.device))
    _lib.check(rc, "lse_combine")
    return (out, lse) if return_lse else out
