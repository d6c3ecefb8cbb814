// Chunked-prefill attention over the paged pool and dense varlen prefill
// (causal, bottom-right aligned), sm_100a.
//
// The reference has no paged prefill: chunks run through HF attention over a
// dense DynamicCache (core/engine.py:1772-1854, core/chunked_prefill.py:9-33),
// and varlen_prefill_attention (core/varlen.py:19-42) wraps
// flash_attn_varlen_func(causal=True) with cu_seqlens_q == cu_seqlens_k.
//
// Design: one CTA = 64 "rows" x one KV head, where the rows pack TQ = 64/n_rep
// query tokens times the n_rep query heads of the group, so each K/V tile is
// read once for the whole GQA group.  K/V tiles of 64 tokens (4 pages) are
// gathered through the block table with 16-byte zero-filling cp.async copies
// into XOR-swizzled shared memory (double buffered).  S = Q K^T and O += P V
// run on mma.m16n8k16 with fp32 accumulation, online softmax in the exp2
// domain; the causal limit of the tile's last query bounds the KV loop.
#include "common.cuh"

namespace bpkv {

struct PrefillTcParams {
  const void* q;
  const void* k;
  const void* v;
  const int32_t* bt;
  const int32_t* cu_q;
  const int32_t* seqlens_k;
  void* out;
  int B, Hq, Hkv, n_rep, tiles_per_req, causal;
  int64_t page_stride, bt_sb;
  float scale_log2;
};
// tcgen05/TMEM kernel (prefill_tc.cu): head_dim 128; BPKV_ERR_UNSUPPORTED otherwise.
int prefill_tc_launch(PrefillTcParams& p, int head_dim, int dtype, int max_seqlen_q, bool paged, cudaStream_t st);

namespace {


constexpr int kRows = 64;   // packed (token, head) rows per CTA
constexpr int kKvTile = 64; // KV tokens per tile
constexpr int kPfWarps = 4;

struct PrefillParams {
  const void* q;
  const void* k;
  const void* v;
  const int32_t* bt;        // paged: [B, max_blocks]
  const int32_t* cu_q;      // [B+1]
  const int32_t* seqlens_k; // paged: [B]; dense: null (== n_q)
  void* out;
  int B, Hq, Hkv, n_rep, max_blocks, tiles_per_req, causal;
  int64_t page_stride, bt_sb;
  float scale_log2;
};

template <typename T, int D, bool PAGED>
__global__ void __launch_bounds__(kPfWarps * 32) prefill_kernel(PrefillParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  constexpr int ROWB = D * 2;
  constexpr int CH = D / 8;
  constexpr int SWM = CH >= 8 ? 7 : CH - 1;
  constexpr int KS = D / 16;
  constexpr int NT = D / 8;
  uint8_t* qs = smem;
  uint8_t* ks = smem + kRows * ROWB;            // 2 buffers
  uint8_t* vs = ks + 2 * kKvTile * ROWB;        // 2 buffers

  const int b = blockIdx.x / p.tiles_per_req;
  const int qt = blockIdx.x % p.tiles_per_req;
  const int hkv = blockIdx.y;
  const int q0 = p.cu_q[b];
  const int nq = p.cu_q[b + 1] - q0;
  const int TQ = kRows / p.n_rep;
  const int tok0 = qt * TQ;
  if (tok0 >= nq) return;
  const int sk = PAGED ? p.seqlens_k[b] : nq;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const T* qg = reinterpret_cast<const T*>(p.q);
  const T* kg = reinterpret_cast<const T*>(p.k);
  const T* vg = reinterpret_cast<const T*>(p.v);

  // ---- Q tile ----
  for (int ci = tid; ci < kRows * CH; ci += blockDim.x) {
    const int m = ci / CH, ch = ci % CH;
    const int tok = tok0 + m / p.n_rep, r = m % p.n_rep;
    const bool ok = tok < nq;
    const T* src = qg + (static_cast<int64_t>(q0 + tok) * p.Hq + hkv * p.n_rep + r) * D + ch * 8;
    cp_async16(smem_u32(qs + m * ROWB + ((ch ^ (m & SWM)) << 4)), ok ? (const void*)src : (const void*)qg, ok);
  }
  const int last_tok = min(tok0 + TQ, nq) - 1;
  int kv_end = sk;
  if (p.causal) kv_end = min(sk, sk - nq + last_tok + 1);
  const int n_tiles = kv_end > 0 ? (kv_end + kKvTile - 1) / kKvTile : 0;

  auto load_kv = [&](int tile, int buf) {
    uint8_t* kb = ks + buf * kKvTile * ROWB;
    uint8_t* vb = vs + buf * kKvTile * ROWB;
    for (int ci = tid; ci < kKvTile * CH; ci += blockDim.x) {
      const int tt = ci / CH, ch = ci % CH;
      const int t = tile * kKvTile + tt;
      const bool ok = t < kv_end;
      int64_t off = 0;
      if (ok) {
        if (PAGED) {
          const int page = __ldg(p.bt + static_cast<int64_t>(b) * p.bt_sb + t / kPage);
          off = static_cast<int64_t>(page) * p.page_stride + (static_cast<int64_t>(t % kPage) * p.Hkv + hkv) * D;
        } else {
          off = (static_cast<int64_t>(q0 + t) * p.Hkv + hkv) * D;
        }
      }
      const uint32_t so = tt * ROWB + ((ch ^ (tt & SWM)) << 4);
      cp_async16(smem_u32(kb + so), ok ? (const void*)(kg + off + ch * 8) : (const void*)kg, ok);
      cp_async16(smem_u32(vb + so), ok ? (const void*)(vg + off + ch * 8) : (const void*)vg, ok);
    }
  };
  if (n_tiles > 0) load_kv(0, 0);
  cp_async_commit();
  cp_async_wait<0>();
  __syncthreads();

  // Q fragments of this warp's 16 rows
  const int mi = lane >> 3, rr = lane & 7, gq = lane >> 2, cq = lane & 3;
  uint32_t qa[KS][4];
#pragma unroll
  for (int kk = 0; kk < KS; ++kk) {
    const int row = warp * 16 + (mi & 1) * 8 + rr;
    const int ch = 2 * kk + (mi >> 1);
    ldmatrix_x4(smem_u32(qs + row * ROWB + ((ch ^ (row & SWM)) << 4)), qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3]);
  }
  // causal limit (absolute kv position) of the lane's two rows
  const int rowA = warp * 16 + gq, rowB = rowA + 8;
  const int tokA = tok0 + rowA / p.n_rep, tokB = tok0 + rowB / p.n_rep;
  const int limA = p.causal ? (tokA < nq ? sk - nq + tokA : sk - 1) : sk - 1;
  const int limB = p.causal ? (tokB < nq ? sk - nq + tokB : sk - 1) : sk - 1;

  float o[NT][4];
#pragma unroll
  for (int n = 0; n < NT; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  float mA = -INFINITY, mB = -INFINITY, lA = 0.f, lB = 0.f;

  for (int it = 0; it < n_tiles; ++it) {
    if (it + 1 < n_tiles) load_kv(it + 1, (it + 1) & 1);
    cp_async_commit();
    if (it > 0) {
      cp_async_wait<1>();
      __syncthreads();
    }
    const uint32_t kb = smem_u32(ks + (it & 1) * kKvTile * ROWB);
    const uint32_t vb = smem_u32(vs + (it & 1) * kKvTile * ROWB);
    float s[8][4];
#pragma unroll
    for (int n = 0; n < 8; ++n) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < KS; ++kk) {
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        const int tt = np * 16 + rr + 8 * (mi >> 1);
        const int ch = 2 * kk + (mi & 1);
        uint32_t b0, b1, b2, b3;
        ldmatrix_x4(kb + tt * ROWB + ((ch ^ (tt & SWM)) << 4), b0, b1, b2, b3);
        mma16816<T>(s[2 * np], qa[kk], b0, b1);
        mma16816<T>(s[2 * np + 1], qa[kk], b2, b3);
      }
    }
    const int tbase = it * kKvTile;
    float mxA = -INFINITY, mxB = -INFINITY;
#pragma unroll
    for (int n = 0; n < 8; ++n) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int t = tbase + n * 8 + 2 * cq + e;
        s[n][e] = t <= limA ? s[n][e] * p.scale_log2 : -INFINITY;
        s[n][2 + e] = t <= limB ? s[n][2 + e] * p.scale_log2 : -INFINITY;
        mxA = fmaxf(mxA, s[n][e]);
        mxB = fmaxf(mxB, s[n][2 + e]);
      }
    }
    mxA = fmaxf(mxA, __shfl_xor_sync(0xffffffffu, mxA, 1));
    mxA = fmaxf(mxA, __shfl_xor_sync(0xffffffffu, mxA, 2));
    mxB = fmaxf(mxB, __shfl_xor_sync(0xffffffffu, mxB, 1));
    mxB = fmaxf(mxB, __shfl_xor_sync(0xffffffffu, mxB, 2));
    const float nA = fmaxf(mA, mxA), nB = fmaxf(mB, mxB);
    // rows with nothing visible yet keep a finite reference point
    const float uA = nA == -INFINITY ? 0.f : nA, uB = nB == -INFINITY ? 0.f : nB;
    const float aA = fast_exp2(mA - uA), aB = fast_exp2(mB - uB);
    mA = nA;
    mB = nB;
    float sumA = 0.f, sumB = 0.f;
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      s[n][0] = fast_exp2(s[n][0] - uA);
      s[n][1] = fast_exp2(s[n][1] - uA);
      s[n][2] = fast_exp2(s[n][2] - uB);
      s[n][3] = fast_exp2(s[n][3] - uB);
      sumA += s[n][0] + s[n][1];
      sumB += s[n][2] + s[n][3];
    }
    lA = lA * aA + sumA;
    lB = lB * aB + sumB;
#pragma unroll
    for (int n = 0; n < NT; ++n) {
      o[n][0] *= aA;
      o[n][1] *= aA;
      o[n][2] *= aB;
      o[n][3] *= aB;
    }
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      uint32_t pa[4], pl[4];
      split2<T>(s[2 * kk][0], s[2 * kk][1], pa[0], pl[0]);
      split2<T>(s[2 * kk][2], s[2 * kk][3], pa[1], pl[1]);
      split2<T>(s[2 * kk + 1][0], s[2 * kk + 1][1], pa[2], pl[2]);
      split2<T>(s[2 * kk + 1][2], s[2 * kk + 1][3], pa[3], pl[3]);
      const int tt = kk * 16 + rr + 8 * (mi & 1);
#pragma unroll
      for (int dt = 0; dt < D / 16; ++dt) {
        const int ch = 2 * dt + (mi >> 1);
        uint32_t b0, b1, b2, b3;
        ldmatrix_x4_trans(vb + tt * ROWB + ((ch ^ (tt & SWM)) << 4), b0, b1, b2, b3);
        mma16816<T>(o[2 * dt], pa, b0, b1);
        mma16816<T>(o[2 * dt + 1], pa, b2, b3);
        if constexpr (SplitP<T>::value) {
          mma16816<T>(o[2 * dt], pl, b0, b1);
          mma16816<T>(o[2 * dt + 1], pl, b2, b3);
        }
      }
    }
    __syncthreads();
  }

  lA += __shfl_xor_sync(0xffffffffu, lA, 1);
  lA += __shfl_xor_sync(0xffffffffu, lA, 2);
  lB += __shfl_xor_sync(0xffffffffu, lB, 1);
  lB += __shfl_xor_sync(0xffffffffu, lB, 2);
  // a row that sees no key (only when seqlen_k < n_q) is written as zeros
  const float invA = lA > 0.f ? 1.f / lA : 0.f, invB = lB > 0.f ? 1.f / lB : 0.f;
  T* og = reinterpret_cast<T*>(p.out);
  if (tokA < nq) {
    T* dst = og + (static_cast<int64_t>(q0 + tokA) * p.Hq + hkv * p.n_rep + rowA % p.n_rep) * D;
#pragma unroll
    for (int n = 0; n < NT; ++n)
      *reinterpret_cast<uint32_t*>(dst + n * 8 + 2 * cq) = pack2<T>(o[n][0] * invA, o[n][1] * invA);
  }
  if (tokB < nq) {
    T* dst = og + (static_cast<int64_t>(q0 + tokB) * p.Hq + hkv * p.n_rep + rowB % p.n_rep) * D;
#pragma unroll
    for (int n = 0; n < NT; ++n)
      *reinterpret_cast<uint32_t*>(dst + n * 8 + 2 * cq) = pack2<T>(o[n][2] * invB, o[n][3] * invB);
  }
}

template <typename T, int D, bool PAGED>
int launch_prefill(PrefillParams& p, int max_seqlen_q, cudaStream_t st) {
  const int TQ = kRows / p.n_rep;
  p.tiles_per_req = (max_seqlen_q + TQ - 1) / TQ;
  if (p.tiles_per_req == 0) return BPKV_OK;
  const size_t smem = static_cast<size_t>(kRows) * D * 2 + 4 * kKvTile * D * 2;
  auto kern = prefill_kernel<T, D, PAGED>;
  static bool raised[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (smem > 48 * 1024 && dev < 64 && !raised[dev]) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) !=
        cudaSuccess) {
      set_error("prefill_launch:smem_attr");
      return BPKV_ERR_CUDA;
    }
    raised[dev] = true;
  }
  dim3 grid(p.B * p.tiles_per_req, p.Hkv);
  kern<<<grid, kPfWarps * 32, smem, st>>>(p);
  BPKV_RETURN_LAUNCH("prefill_launch");
}

template <bool PAGED>
int try_tc(const PrefillParams& p, int D, int dtype, int max_seqlen_q, cudaStream_t st) {
  PrefillTcParams t{};
  t.q = p.q;
  t.k = p.k;
  t.v = p.v;
  t.bt = p.bt;
  t.cu_q = p.cu_q;
  t.seqlens_k = p.seqlens_k;
  t.out = p.out;
  t.B = p.B;
  t.Hq = p.Hq;
  t.Hkv = p.Hkv;
  t.n_rep = p.n_rep;
  t.causal = p.causal;
  t.page_stride = p.page_stride;
  t.bt_sb = p.bt_sb;
  t.scale_log2 = p.scale_log2;
  return prefill_tc_launch(t, D, dtype, max_seqlen_q, PAGED, st);
}

template <bool PAGED>
int dispatch_prefill(PrefillParams& p, int D, int dtype, int max_seqlen_q, cudaStream_t st) {
  const int rc = try_tc<PAGED>(p, D, dtype, max_seqlen_q, st);
  if (rc != BPKV_ERR_UNSUPPORTED) return rc;
#define BPKV_PF(TY)                                                              \
  switch (D) {                                                                   \
    case 64: return launch_prefill<TY, 64, PAGED>(p, max_seqlen_q, st);          \
    case 128: return launch_prefill<TY, 128, PAGED>(p, max_seqlen_q, st);        \
    default: return launch_prefill<TY, 256, PAGED>(p, max_seqlen_q, st);         \
  }
  if (dtype == BPKV_BF16) {
    BPKV_PF(__nv_bfloat16)
  } else {
    BPKV_PF(__half)
  }
#undef BPKV_PF
}

int check_common(int batch, int Hq, int Hkv, int D, int dtype, const void* q, const void* k, const void* v,
                 void* out) {
  BPKV_CHECK_ARG(batch >= 0 && Hq > 0 && Hkv > 0 && Hq % Hkv == 0, "prefill_shape_unsupported:gqa");
  BPKV_CHECK_ARG(64 % (Hq / Hkv) == 0, "prefill_shape_unsupported:gqa_ratio_%d", Hq / Hkv);
  BPKV_CHECK_ARG(q && k && v && out, "prefill_shape_unsupported:null_pointer");
  if (!(D == 64 || D == 128 || D == 256) || (dtype != BPKV_BF16 && dtype != BPKV_F16)) {
    set_error("prefill_shape_unsupported:head_dim_%d_dtype_%d", D, dtype);
    return BPKV_ERR_UNSUPPORTED;
  }
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out)) {
    set_error("prefill_shape_unsupported:alignment");
    return BPKV_ERR_UNSUPPORTED;
  }
  return BPKV_OK;
}

}  // namespace
}  // namespace bpkv

using namespace bpkv;

extern "C" BPKV_API int bpkv_paged_prefill(const void* q, const void* k_cache, const void* v_cache,
                                           const int32_t* block_table, const int32_t* cu_seqlens_q,
                                           const int32_t* seqlens_k, void* out, int batch, int num_q_heads,
                                           int num_kv_heads, int head_dim, int max_blocks, int max_seqlen_q,
                                           int64_t page_stride, int64_t bt_stride_b, float softmax_scale,
                                           int causal, int dtype, void* stream) {
  clear_error();
  int rc = check_common(batch, num_q_heads, num_kv_heads, head_dim, dtype, q, k_cache, v_cache, out);
  if (rc != BPKV_OK) return rc;
  BPKV_CHECK_ARG(block_table && cu_seqlens_q && seqlens_k, "prefill_shape_unsupported:null_pointer");
  BPKV_CHECK_ARG(page_stride % 8 == 0, "prefill_shape_unsupported:page_stride");
  if (batch == 0 || max_seqlen_q <= 0) return BPKV_OK;
  PrefillParams p{};
  p.q = q;
  p.k = k_cache;
  p.v = v_cache;
  p.bt = block_table;
  p.cu_q = cu_seqlens_q;
  p.seqlens_k = seqlens_k;
  p.out = out;
  p.B = batch;
  p.Hq = num_q_heads;
  p.Hkv = num_kv_heads;
  p.n_rep = num_q_heads / num_kv_heads;
  p.max_blocks = max_blocks;
  p.causal = causal;
  p.page_stride = page_stride;
  p.bt_sb = bt_stride_b;
  p.scale_log2 = softmax_scale * 1.4426950408889634f;
  return dispatch_prefill<true>(p, head_dim, dtype, max_seqlen_q, static_cast<cudaStream_t>(stream));
}

extern "C" BPKV_API int bpkv_varlen_prefill(const void* q, const void* k, const void* v,
                                            const int32_t* cu_seqlens, void* out, int batch, int num_q_heads,
                                            int num_kv_heads, int head_dim, int max_seqlen, float softmax_scale,
                                            int causal, int dtype, void* stream) {
  clear_error();
  int rc = check_common(batch, num_q_heads, num_kv_heads, head_dim, dtype, q, k, v, out);
  if (rc != BPKV_OK) return rc;
  BPKV_CHECK_ARG(cu_seqlens != nullptr, "prefill_shape_unsupported:null_pointer");
  if (batch == 0 || max_seqlen <= 0) return BPKV_OK;
  PrefillParams p{};
  p.q = q;
  p.k = k;
  p.v = v;
  p.cu_q = cu_seqlens;
  p.out = out;
  p.B = batch;
  p.Hq = num_q_heads;
  p.Hkv = num_kv_heads;
  p.n_rep = num_q_heads / num_kv_heads;
  p.causal = causal;
  p.scale_log2 = softmax_scale * 1.4426950408889634f;
  return dispatch_prefill<false>(p, head_dim, dtype, max_seqlen, static_cast<cudaStream_t>(stream));
}
