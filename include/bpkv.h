/*
 * bpkv.h — C ABI of libbpkv.so, the B200 (sm_100a) kernels behind the
 * block-paged KV hot path of BP-KV (majic-mk/UnifiedKV).
 *
 * Conventions for every entry point:
 *   - Pointers are raw device pointers unless stated otherwise; sizes and
 *     strides are in ELEMENTS of the stated dtype (not bytes).
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy default stream).
 *     Every call is asynchronous on that stream; nothing synchronises.
 *   - The return value is BPKV_OK (0) or an error code below; a human readable
 *     reason for the last failure on the calling thread is available from
 *     bpkv_last_error().  Shape errors are reported with the same reason tokens
 *     the reference raises (e.g. "page16_native_shape_unsupported:gqa").
 *   - dtype codes: BPKV_F32, BPKV_F16, BPKV_BF16.
 *   - Paged KV layout (reference core/pool.py:20-71, one layer's view):
 *       cache[page][token 0..15][kv_head][head_dim], the token/head/dim part of a
 *       page contiguous; `page_stride` is the distance between pages.
 *   - No call allocates device memory except where "workspace" is documented
 *     as caller-provided: the caller sizes it with the matching *_workspace_size.
 */
#ifndef BPKV_H
#define BPKV_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define BPKV_API __attribute__((visibility("default")))
#else
#define BPKV_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

enum {
  BPKV_OK = 0,
  BPKV_ERR_SHAPE = 1,       /* shape / argument rejected (reference error token) */
  BPKV_ERR_UNSUPPORTED = 2, /* valid but not supported by this build            */
  BPKV_ERR_CUDA = 3,        /* CUDA runtime error (launch / config)             */
  BPKV_ERR_WORKSPACE = 4    /* workspace missing or too small                   */
};

enum { BPKV_F32 = 0, BPKV_F16 = 1, BPKV_BF16 = 2 };

/* Reason string for the last non-zero return on this thread ("" if none). */
BPKV_API const char* bpkv_last_error(void);

/* Library version (major*10000 + minor*100 + patch). */
BPKV_API int bpkv_version(void);

/* Hash of the sources the library was built from (16 hex digits; build.py's
 * tree_hash over csrc/*.cu, csrc/*.cuh, include/*.h).  The Python loader refuses
 * a library whose hash differs from the tree it sits in. */
BPKV_API const char* bpkv_build_hash(void);

/* Number of streaming multiprocessors of the current device (cached per device). */
BPKV_API int bpkv_num_sms(void);

/* Diagnostics (no counterpart in the reference): a launch of `blocks` CTAs of 256
 * threads that evaluate bpkv_debug_exp2_count(blocks, iters) hardware exp2 (the
 * ex2.approx instruction of the scoring and softmax kernels) in independent
 * chains; time it with CUDA events to get this GPU's exp2 rate.  sink: any
 * device float (never written in practice). */
BPKV_API int bpkv_debug_exp2_rate(int blocks, int iters, float* sink, void* stream);
BPKV_API long long bpkv_debug_exp2_count(int blocks, int iters);

/* ------------------------------------------------------------------------ *
 * Page16 decode attention.
 * Replaces page16_decode_attention / _page16_decode_kernel
 * (core/page16_native.py:83-150, kernel :17-80) and the gather-then-attention
 * rebuild path (core/engine.py:4060-4100) it stands in for.
 *
 *   out[b,h,:] = softmax(scale * q[b,h,:] . K[b, t, h / n_rep, :], t < len_b) . V
 *   with K/V rows of request b at page block_table[b, t / 16], row t % 16, and
 *   len_b = min(cache_seqlens[b], 16 * max_blocks)  (pages past max_blocks are
 *   never read, as in the reference loop).  len_b <= 0 yields NaN rows, as the
 *   reference's 0/0 does.
 *
 * q:            [batch, num_q_heads, head_dim], strides (q_stride_b, q_stride_h), unit dim stride
 * k/v_cache:    paged layout above, stride between pages = page_stride
 * block_table:  int32 [batch, max_blocks], row stride bt_stride_b
 * cache_seqlens:int32 [batch], lengths INCLUDING the current token
 * out:          [batch, num_q_heads, head_dim] contiguous, same dtype as q
 * lse_out:      optional fp32 [batch, num_q_heads]: natural-log sum-exp of the
 *               scaled logits (for cross-GPU merges); may be NULL
 * workspace:    device scratch of bpkv_page16_decode_workspace_size() bytes
 * ------------------------------------------------------------------------ */
BPKV_API size_t bpkv_page16_decode_workspace_size(int batch, int num_q_heads, int num_kv_heads,
                                         int head_dim, int dtype);

BPKV_API int bpkv_page16_decode(const void* q, const void* k_cache, const void* v_cache,
                       const int32_t* block_table, const int32_t* cache_seqlens,
                       void* out, float* lse_out,
                       int batch, int num_q_heads, int num_kv_heads, int head_dim,
                       int max_blocks, int64_t q_stride_b, int64_t q_stride_h,
                       int64_t page_stride, int64_t bt_stride_b,
                       float softmax_scale, int dtype,
                       void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------ *
 * Page16 decode with the decode-token append fused in.
 * Replaces the pair "scatter the new k/v into the pool page, then
 * page16_decode_attention" of direct_forward (core/scheduler.py:398-418).
 * cache_seqlens include the new token (the reference passes lens+1); the new
 * token's row k_new/v_new[b] ([batch, num_kv_heads, head_dim], row stride
 * new_stride_b) is written to the pool at (block_table[b, (len-1)/16],
 * (len-1) % 16) and used by the same launch.  Requests whose length exceeds
 * 16*max_blocks are decoded without the append.  Other arguments as
 * bpkv_page16_decode.
 * ------------------------------------------------------------------------ */
BPKV_API int bpkv_page16_decode_append(const void* q, const void* k_new, const void* v_new,
                       int64_t new_stride_b, void* k_cache, void* v_cache,
                       const int32_t* block_table, const int32_t* cache_seqlens,
                       void* out, float* lse_out,
                       int batch, int num_q_heads, int num_kv_heads, int head_dim,
                       int max_blocks, int64_t q_stride_b, int64_t q_stride_h,
                       int64_t page_stride, int64_t bt_stride_b,
                       float softmax_scale, int dtype,
                       void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------ *
 * Allocation-free Page16 decode.  No counterpart in the reference: this entry
 * point exists for callers of this library that cannot allocate device memory
 * when they decode - an engine that reserved nearly all of HBM for the paged
 * pool up front, a non-Python host binding this C ABI without a device
 * allocator, or a latency-critical loop that must avoid cudaMalloc's implicit
 * synchronisation.  Same arguments and results as bpkv_page16_decode minus
 * the workspace: the scratch is a file-scope device array of
 * bpkv_page16_decode_noalloc_max_scratch() bytes (16 MiB), held by every GPU
 * that loads the library until exit.  Shapes whose scratch
 * (bpkv_page16_decode_workspace_size) exceeds it are rejected with
 * BPKV_ERR_WORKSPACE.  The first call on a device looks up the array's device
 * address (cudaGetSymbolAddress) and should come before any stream capture;
 * the address is kept per device index for the life of the process, so after
 * cudaDeviceReset (or under another context on that device) it is stale and
 * this entry point must not be called again there.
 * All calls share the array: calls that overlap on the GPU race and must be
 * serialised by the caller.  It calls no cudaMalloc / cudaFree.
 * ------------------------------------------------------------------------ */
BPKV_API size_t bpkv_page16_decode_noalloc_max_scratch(void);

BPKV_API int bpkv_page16_decode_noalloc(const void* q, const void* k_cache, const void* v_cache,
                       const int32_t* block_table, const int32_t* cache_seqlens,
                       void* out, float* lse_out,
                       int batch, int num_q_heads, int num_kv_heads, int head_dim,
                       int max_blocks, int64_t q_stride_b, int64_t q_stride_h,
                       int64_t page_stride, int64_t bt_stride_b,
                       float softmax_scale, int dtype, void* stream);

/* ------------------------------------------------------------------------ *
 * Log-sum-exp merge of partial attention results (split-KV across GPUs).
 * The reference has no counterpart: it never splits a sequence across GPUs
 * (core/multi_gpu.py:7-123 only mirrors KV-head shards).  This merge completes
 * the split-KV path that replaces that mirror.
 *
 * part_out: fp32 [num_parts, rows, head_dim]; part_lse: fp32 [num_parts, rows]
 * out: [rows, head_dim] in out_dtype; lse_out: optional fp32 [rows].
 * A part whose lse is -inf contributes nothing; all parts -inf -> NaN row.
 * ------------------------------------------------------------------------ */
BPKV_API int bpkv_lse_combine(const float* part_out, const float* part_lse, void* out, float* lse_out,
                     int num_parts, int rows, int head_dim, int out_dtype, void* stream);

/* ------------------------------------------------------------------------ *
 * Split-KV merge over NVLink peer memory.
 * Replaces the all-gather of packed (out, lse) partials + merge of the
 * long-sequence decode (the reference mirrors KV heads between GPUs instead,
 * core/multi_gpu.py:7-123; this build splits one sequence's pages across
 * GPUs).  Setup, once per process group and shape:
 *   bytes = bpkv_peer_exchange_bytes(world, rows, head_dim);
 *   bpkv_peer_buffer_alloc(bytes, &own, handle)   (zeroed; 64-byte CUDA IPC handle)
 *   exchange the handles between the processes, then on every rank
 *   bpkv_peer_buffer_open(handle_of_rank_r, &bufs[r]) for r != rank (bufs[rank] = own).
 * Per call (every rank makes the same sequence of calls; the call number is
 * kept in the buffer itself, so the call's kernel can be captured in a CUDA
 * graph and replayed):
 *   bpkv_split_kv_merge_p2p: this rank's partial part_out [rows, head_dim]
 *   (dtype) with natural-log part_lse [rows] is stored into every rank's
 *   buffer over NVLink as 16-byte words of two 64-bit halves, each an fp32
 *   value beside the call number (no separate flag or fence), then every rank
 *   polls the words of this call and writes the merged out [rows, head_dim]
 *   in out_dtype (and lse_out [rows] if not null).  The launch is a programmatic dependent
 *   launch: it may start during the grid that produced part_out and waits
 *   for it.  A wait gives up after max_polls polls (or 4 s): *status is set
 *   to 1 and the rows are NaN.
 * Teardown: bpkv_peer_buffer_close(bufs[r]) for r != rank, after a barrier
 * bpkv_peer_buffer_free(own).  world <= 8; head_dim % 4 == 0.  No multicast.
 * ------------------------------------------------------------------------ */
BPKV_API size_t bpkv_peer_exchange_bytes(int world, int rows, int head_dim);
BPKV_API int bpkv_peer_buffer_alloc(size_t bytes, void** ptr, void* ipc_handle);
BPKV_API int bpkv_peer_buffer_open(const void* ipc_handle, void** ptr);
BPKV_API int bpkv_peer_buffer_close(void* ptr);
BPKV_API int bpkv_peer_buffer_free(void* ptr);
BPKV_API int bpkv_split_kv_merge_p2p(const void* part_out, const float* part_lse, void* const* peer_bufs,
                     int rank, int world, int rows, int head_dim, uint32_t max_polls,
                     void* out, float* lse_out, int* status, int dtype, int out_dtype, void* stream);

/* ------------------------------------------------------------------------ *
 * Split-KV decode of sequences whose pages are split across GPUs, with the
 * exchange fused into the combine.  Replaces, for one long sequence, the
 * reference's multi-GPU decode (core/multi_gpu.py:7-123 mirrors KV heads and
 * decode falls back to a dense rebuild, core/engine.py:2841-2851).
 * Arguments up to workspace_bytes are those of bpkv_page16_decode, for THIS
 * rank's page range (block table and token counts of the range), except that
 * out is [batch, num_q_heads, head_dim] in out_dtype (dtype, or BPKV_F32).
 * Two launches: the decode grid (num_splits CTAs over the flattened page list,
 * 0 = one per SM) leaves an fp32 partial per CTA; a programmatic dependent
 * kernel, one CTA per (request, q-head) row, merges the row's partials in fp32,
 * stores the rank's (o, lse) into every peer's exchange buffer (peer_bufs as
 * for bpkv_split_kv_merge_p2p, rows = batch * num_q_heads; may be NULL when
 * world == 1), polls the peers' words of this call and writes the merged row
 * once (lse_out optional, natural log).  No partial is rounded to a 16-bit
 * type before the final merge.  Rows with no keys on any rank are NaN (lse
 * -inf).  A wait gives up after max_polls polls (or 4 s): *status = 1 and the
 * row is NaN.  world <= 8; head_dim % 4 == 0.  No multicast.
 * ------------------------------------------------------------------------ */
BPKV_API int bpkv_split_kv_decode_p2p(const void* q, const void* k_cache, const void* v_cache,
                     const int32_t* block_table, const int32_t* cache_seqlens, void* out,
                     float* lse_out, int batch, int num_q_heads, int num_kv_heads, int head_dim,
                     int max_blocks, int64_t q_stride_b, int64_t q_stride_h, int64_t page_stride,
                     int64_t bt_stride_b, float softmax_scale, int dtype, int out_dtype,
                     void* workspace, size_t workspace_bytes, int num_splits,
                     void* const* peer_bufs, int rank, int world, uint32_t max_polls,
                     int* status, void* stream);

/* ------------------------------------------------------------------------ *
 * Decode-token append: writes this step's k/v into the paged pool at slot
 * (block_table[b, old_len/16], old_len % 16).
 * Replaces the indexed scatter of core/scheduler.py:398-408
 * (pool.write_one_token, core/pool.py:143-152).
 * k_new/v_new: [batch, num_kv_heads, head_dim], row stride new_stride_b.
 * Requests with old_len < 0 or old_len >= 16*max_blocks are skipped.
 * ------------------------------------------------------------------------ */
BPKV_API int bpkv_decode_append(const void* k_new, const void* v_new, void* k_cache, void* v_cache,
                       const int32_t* block_table, const int32_t* old_lens,
                       int batch, int num_kv_heads, int head_dim, int max_blocks,
                       int64_t new_stride_b, int64_t page_stride, int64_t bt_stride_b,
                       int dtype, void* stream);

/* ------------------------------------------------------------------------ *
 * Observation-window block scoring (fused: the [h_q, window, T] attention
 * matrix is never materialised).
 * Replaces KVScheduler._score_layer_blocks_for_selection
 * (core/scheduler.py:565-592) and the score part of BlockAlignedSnapKV.compress
 * (core/compress.py:100-130):
 *   K_mid = K[:, sink_len : L - obs_len, :] zero-padded to N*16 tokens,
 *   A = softmax(scale * Q_obs . K_mid^T) over all N*16 tokens (pad included),
 *   S[t] = max_h mean_i A[h, i, t];  block[n] = sum_{t in block n} S[t];
 *   if smooth and N >= 3: block = max_pool1d(block, 3, stride 1, pad 1).
 *
 * k:      [num_kv_heads, L, head_dim]   strides (k_stride_h, k_stride_t)
 * q_obs:  [num_q_heads, window, head_dim] strides (q_stride_h, q_stride_t)
 * block_scores: fp32 [N], N = ceil((L - sink_len - obs_len) / 16)
 * workspace: bpkv_block_score_workspace_size() bytes
 * Precondition (reference): L >= sink_len + obs_len + 16, else BPKV_ERR_SHAPE.
 * ------------------------------------------------------------------------ */
BPKV_API size_t bpkv_block_score_workspace_size(int num_q_heads, int window, int L, int sink_len,
                                       int obs_len);

BPKV_API int bpkv_block_score(const void* k, const void* q_obs, float* block_scores,
                     int num_kv_heads, int num_q_heads, int L, int window, int head_dim,
                     int sink_len, int obs_len,
                     int64_t k_stride_h, int64_t k_stride_t,
                     int64_t q_stride_h, int64_t q_stride_t,
                     float softmax_scale, int smooth, int dtype,
                     void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------ *
 * Per-KV-head block scores (the "top 25% of blocks per KV head" reading of
 * the compression benchmark).  The reference has no such mode: its score is
 * shared across KV heads (max over all q heads, core/compress.py:116-130,
 * core/scheduler.py:565-592).  Here KV head g keeps its own row
 *   S_g[t] = max_{h in group g} mean_i A[h, i, t],  block_g[n] = sum_t S_g[t],
 * smoothed per row as above.  block_scores: fp32 [num_kv_heads][N].  Other
 * arguments and the workspace as bpkv_block_score.
 * ------------------------------------------------------------------------ */
BPKV_API int bpkv_block_score_per_kv_head(const void* k, const void* q_obs, float* block_scores,
                     int num_kv_heads, int num_q_heads, int L, int window, int head_dim,
                     int sink_len, int obs_len,
                     int64_t k_stride_h, int64_t k_stride_t,
                     int64_t q_stride_h, int64_t q_stride_t,
                     float softmax_scale, int smooth, int dtype,
                     void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------ *
 * Deterministic top-k block selection.
 * Replaces torch.topk + sort (core/compress.py:140-142) and
 * torch.topk + sorted(set(...)) (core/scheduler.py:615-616); ties are broken by
 * the LOWEST block index (torch leaves tie order unspecified).
 * scores: fp32 [n]; selected: int32 [k] written in ascending index order.
 * n <= 49152.  NaN scores rank above every number (as torch.topk).
 * ------------------------------------------------------------------------ */
BPKV_API int bpkv_topk_select(const float* scores, int n, int k, int32_t* selected, void* stream);

/* Batched form: rows b = 0..batch-1 of scores [batch][n] -> selected
 * [batch][k], one independent selection per row (per-KV-head mode: one row
 * per KV head).  Same rules as bpkv_topk_select; no reference counterpart. */
BPKV_API int bpkv_topk_select_batched(const float* scores, int n, int k, int batch, int32_t* selected,
                     void* stream);

/* ------------------------------------------------------------------------ *
 * Compacting writeback of one layer into freshly allocated pool pages.
 * Replaces _write_selected_layer_to_pool / _write_block_indexed_layer_to_pool /
 * _write_piece_to_blocks (core/scheduler.py:666-799).  Destination token p of
 * the compacted sequence (effective_len = sink + 16*k + obs tokens) reads:
 *   p <  sink                      : source token p
 *   sink <= p < sink + 16k         : r=(p-sink)/16, o=(p-sink)%16,
 *                                    source sink + 16*selected[r] + o, zero if
 *                                    that lies at or past L - obs (padding)
 *   p >= sink + 16k                : source L - obs + (p - sink - 16k)
 * With k_blocks < 0 the layer is copied uncompressed: p -> p for p < L
 * (the "input_le_budget"/"too_short" modes).  Slots of the last page past
 * effective_len are left untouched, as in the reference.
 * k_src/v_src: [num_kv_heads, L, head_dim] strides (src_stride_h, src_stride_t)
 * dst_pages:   int32 [ceil(effective_len/16)] destination page ids
 * k/v_dst:     destination; element (page, slot, head, dim) lives at
 *              page*page_stride + slot*dst_stride_t + head*dst_stride_h + dim.
 *              A pool layer view is (page_stride, h_kv*d, d); a dense
 *              [h_kv, effective_len, d] tensor is (16*d, d, effective_len*d)
 *              with dst_pages = 0, 1, 2, ...
 * ------------------------------------------------------------------------ */
BPKV_API int bpkv_page_compact(const void* k_src, const void* v_src, void* k_dst, void* v_dst,
                      const int32_t* selected, int k_blocks, const int32_t* dst_pages,
                      int L, int sink_len, int obs_len, int num_kv_heads, int head_dim,
                      int64_t src_stride_h, int64_t src_stride_t, int64_t page_stride,
                      int64_t dst_stride_t, int64_t dst_stride_h, int dtype, void* stream);

/* Per-KV-head compaction: KV head h takes its mid blocks from
 * selected + h * selected_stride_h (int32 [num_kv_heads][>= k_blocks], ascending
 * per head), so every head keeps its own blocks in the same destination pages;
 * all heads share the effective length.  Decode over such pages is unchanged
 * (keys already carry their positions through RoPE).  Other arguments as
 * bpkv_page_compact.  No reference counterpart (its selection is shared
 * across KV heads, core/scheduler.py:735-799). */
BPKV_API int bpkv_page_compact_per_kv_head(const void* k_src, const void* v_src, void* k_dst, void* v_dst,
                     const int32_t* selected, int64_t selected_stride_h, int k_blocks,
                     const int32_t* dst_pages, int L, int sink_len, int obs_len,
                     int num_kv_heads, int head_dim,
                     int64_t src_stride_h, int64_t src_stride_t,
                     int64_t page_stride, int64_t dst_stride_t, int64_t dst_stride_h,
                     int dtype, void* stream);

/* ------------------------------------------------------------------------ *
 * Paged chunked-prefill attention (causal, bottom-right aligned).
 * New path: the reference runs chunks through HF attention over a dense
 * DynamicCache (core/engine.py:1772-1854, core/chunked_prefill.py:9-33) and
 * only wraps flash_attn_varlen_func for the no-past case (core/varlen.py:19-42).
 * Request b has q rows cu_seqlens_q[b] .. cu_seqlens_q[b+1]-1 (n_q of them)
 * attending to its first seqlens_k[b] KV tokens (paged via block_table, the
 * chunk's own K/V already written to the pool); query i of the chunk sees
 * tokens t <= seqlens_k[b] - n_q + i.
 * q/out: [total_q, num_q_heads, head_dim] contiguous.
 * ------------------------------------------------------------------------ */
BPKV_API int bpkv_paged_prefill(const void* q, const void* k_cache, const void* v_cache,
                       const int32_t* block_table, const int32_t* cu_seqlens_q,
                       const int32_t* seqlens_k, void* out,
                       int batch, int num_q_heads, int num_kv_heads, int head_dim,
                       int max_blocks, int max_seqlen_q, int64_t page_stride,
                       int64_t bt_stride_b, float softmax_scale, int causal, int dtype,
                       void* stream);

/* ------------------------------------------------------------------------ *
 * Dense varlen prefill attention (no past context): cu_seqlens_q == cu_seqlens_k.
 * Replaces varlen_prefill_attention (core/varlen.py:19-42), which calls
 * flash_attn_varlen_func(causal=True).
 * q: [total, num_q_heads, head_dim]; k/v: [total, num_kv_heads, head_dim]
 * (contiguous); out like q.
 * ------------------------------------------------------------------------ */
BPKV_API int bpkv_varlen_prefill(const void* q, const void* k, const void* v,
                        const int32_t* cu_seqlens, void* out,
                        int batch, int num_q_heads, int num_kv_heads, int head_dim,
                        int max_seqlen, float softmax_scale, int causal, int dtype,
                        void* stream);

/* ------------------------------------------------------------------------ *
 * Batched page gather / scatter between the pool and a packed staging buffer
 * (offload / prefetch of cold pages).  Replaces the per-block copies of
 * AsyncOffloadManager._read/_write_single_block_* (core/offload.py:163-179,
 * 577-599, 662-691).  packed: [n_pages, page_elems] contiguous, page_elems =
 * 16 * num_kv_heads * head_dim.  Either side may be pinned host memory that is
 * mapped into the device address space.
 * ------------------------------------------------------------------------ */
BPKV_API int bpkv_page_gather(const void* pool, const int32_t* page_ids, int n_pages, void* packed,
                     int64_t page_elems, int64_t page_stride, int dtype, void* stream);
BPKV_API int bpkv_page_scatter(const void* packed, const int32_t* page_ids, int n_pages, void* pool,
                      int64_t page_elems, int64_t page_stride, int dtype, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* BPKV_H */
