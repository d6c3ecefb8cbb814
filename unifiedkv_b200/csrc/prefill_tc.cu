// Paged chunked-prefill / varlen attention on the 5th-generation tensor cores
// (tcgen05.mma with TMEM accumulators), sm_100a, head_dim 128, bf16 / fp16.
//
// Same semantics as prefill.cu (causal, bottom-right aligned; K/V gathered
// from 16-token pages through the block table, or dense varlen).  Per CTA:
//   * 128 accumulator rows = 128/n_rep query tokens x the n_rep query heads of
//     one KV head (a GQA group shares every K/V tile), 4 warps, thread i owns
//     row i (= TMEM lane i), so the softmax needs no shuffles;
//   * K/V tiles of 64 tokens are gathered with 16-byte cp.async into the
//     128-byte-swizzled layout the UMMA descriptors describe
//     ([64-column block][token][128 B], chunk ^= row & 7, 1024-byte aligned),
//     double buffered; Q uses the same layout;
//   * S = Q K^T: one elected thread issues 8 tcgen05.mma (M128 N64 K16, both
//     operands K-major) into TMEM columns [0,64), commit -> mbarrier;
//   * the 128 threads pull their S row with tcgen05.ld, apply the causal mask
//     and online softmax (exp2 domain) and store P to shared memory as
//     bf16 hi + lo parts (fp16: one part) in the K-major swizzled layout;
//   * O_tile = P V: tcgen05.mma M128 N128 K16 with V as an MN-major operand
//     (the same [64-d block][token] tiles), into TMEM columns [64,192);
//     threads fold it into register accumulators with the softmax rescale.
// Every mbarrier wait is bounded; on a timeout the CTA abandons its tile,
// writes NaN rows and still frees its TMEM.
#include "common.cuh"
#include "tcgen05.cuh"

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

namespace {

constexpr int kD = 128, kBM = 128, kBN = 64, kDB = kD / 64;
constexpr int kQBytes = kDB * kBM * 128;       // 32 KB
constexpr int kKVBytes = kDB * kBN * 128;      // 16 KB per K or V tile
constexpr int kPBytes = kBM * 128;             // 16 KB (64 tokens per row)
constexpr int kNBuf = 4;                       // K/V ring depth
constexpr int kSmemBytes = kQBytes + 2 * kNBuf * kKVBytes + 2 * kPBytes + 1024 /*align*/ + 64;
constexpr uint32_t kTmemCols = 512;            // S0 [0,64) S1 [64,128) O0 [128,256) O1 [256,384)

__device__ __forceinline__ uint32_t sw_off(int row, int chunk) {  // chunk 0..7 inside a 128-B row
  return static_cast<uint32_t>(row * 128 + ((chunk ^ (row & 7)) << 4));
}

template <typename T, bool PAGED>
__global__ void __launch_bounds__(128, 1) prefill_tc_kernel(PrefillTcParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* qs = smem;
  uint8_t* ks = qs + kQBytes;            // kNBuf buffers
  uint8_t* vs = ks + kNBuf * kKVBytes;   // kNBuf buffers
  uint8_t* ph = vs + kNBuf * kKVBytes;
  uint8_t* pl = ph + kPBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(pl + kPBytes);  // S0, S1, O0, O1
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 4);

  const int b = blockIdx.x / p.tiles_per_req;
  const int qt = blockIdx.x % p.tiles_per_req;
  const int hkv = blockIdx.y;
  const int q0 = p.cu_q[b];
  const int nq = p.cu_q[b + 1] - q0;
  const int TQ = kBM / p.n_rep;
  const int tok0 = qt * TQ;
  if (tok0 >= nq) return;  // uniform across the CTA: before any barrier or TMEM use
  const int sk = PAGED ? p.seqlens_k[b] : nq;
  const int tid = threadIdx.x, warp = tid >> 5;
  const T* qg = reinterpret_cast<const T*>(p.q);
  const T* kg = reinterpret_cast<const T*>(p.k);
  const T* vg = reinterpret_cast<const T*>(p.v);

  if (warp == 0) {
    tc::tmem_alloc(smem_u32(tmem_slot), kTmemCols);
    tc::tmem_relinquish();
  }
  if (tid == 0) {
    for (int i = 0; i < 4; ++i) tc::mbar_init(smem_u32(&bars[i]), 1);
    tc::fence_mbar_init();
  }

  // ---- Q tile: row m = (token tok0 + m / n_rep, head m % n_rep) ----
  for (int ci = tid; ci < kBM * (kD / 8); ci += 128) {
    const int m = ci / (kD / 8), ch = ci % (kD / 8);
    const int tok = tok0 + m / p.n_rep, r = m % p.n_rep;
    const bool ok = tok < nq;
    const T* src = qg + (static_cast<int64_t>(q0 + tok) * p.Hq + hkv * p.n_rep + r) * kD + ch * 8;
    cp_async16(smem_u32(qs + (ch >> 3) * (kBM * 128) + sw_off(m, ch & 7)), ok ? (const void*)src : (const void*)qg, ok);
  }
  const int last_tok = min(tok0 + TQ, nq) - 1;
  const int kv_end = p.causal ? min(sk, sk - nq + last_tok + 1) : sk;
  const int n_tiles = kv_end > 0 ? (kv_end + kBN - 1) / kBN : 0;

  auto load_kv = [&](int tile, int buf) {
    uint8_t* kb = ks + buf * kKVBytes;
    uint8_t* vb = vs + buf * kKVBytes;
    for (int ci = tid; ci < kBN * (kD / 8); ci += 128) {
      const int tt = ci / (kD / 8), ch = ci % (kD / 8);
      const int t = tile * kBN + tt;
      const bool ok = t < kv_end;
      int64_t off = 0;
      if (ok) {
        if (PAGED) {
          const int page = __ldg(p.bt + static_cast<int64_t>(b) * p.bt_sb + t / kPage);
          off = static_cast<int64_t>(page) * p.page_stride + (static_cast<int64_t>(t % kPage) * p.Hkv + hkv) * kD;
        } else {
          off = (static_cast<int64_t>(q0 + t) * p.Hkv + hkv) * kD;
        }
      }
      const uint32_t so = (ch >> 3) * (kBN * 128) + sw_off(tt, ch & 7);
      cp_async16(smem_u32(kb + so), ok ? (const void*)(kg + off + ch * 8) : (const void*)kg, ok);
      cp_async16(smem_u32(vb + so), ok ? (const void*)(vg + off + ch * 8) : (const void*)vg, ok);
    }
  };
  // prologue: tiles 0..2 in flight (one commit group per tile, empty groups past the end)
#pragma unroll
  for (int t = 0; t < kNBuf - 1; ++t) {
    if (t < n_tiles) load_kv(t, t);
    cp_async_commit();
  }

  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
  constexpr bool kBf16 = SplitP<T>::value;
  const uint32_t id_s = tc::idesc_f16(kBf16, false, false, kBM, kBN);
  const uint32_t id_o = tc::idesc_f16(kBf16, false, true, kBM, kD);
  auto t_s = [&](int j) { return tmem + static_cast<uint32_t>((j & 1) * kBN); };
  auto t_o = [&](int j) { return tmem + 2u * kBN + static_cast<uint32_t>((j & 1) * kD); };
  auto bar_s = [&](int j) { return smem_u32(&bars[j & 1]); };
  auto bar_o = [&](int j) { return smem_u32(&bars[2 + (j & 1)]); };

  // row of this thread
  const int row = tid;
  const int tok = tok0 + row / p.n_rep;
  const int lim = p.causal ? (tok < nq ? sk - nq + tok : sk - 1) : sk - 1;
  float acc[kD];
#pragma unroll
  for (int i = 0; i < kD; ++i) acc[i] = 0.f;
  float m_run = -INFINITY, l_run = 0.f, alpha_prev = 1.f;
  bool failed = false;

  // S(j) = Q K(j)^T into S buffer j&1 (issued by one thread)
  auto issue_s = [&](int j) {
    tc::tc_fence_after();
    const uint32_t qa = smem_u32(qs), kb = smem_u32(ks + (j % kNBuf) * kKVBytes);
#pragma unroll
    for (int kk = 0; kk < kD / 16; ++kk) {
      const uint32_t koff = (kk & 3) * 32;
      const uint64_t ad = tc::smem_desc_sw128(qa + (kk >> 2) * (kBM * 128) + koff, 16, 1024);
      const uint64_t bd = tc::smem_desc_sw128(kb + (kk >> 2) * (kBN * 128) + koff, 16, 1024);
      tc::mma_f16(t_s(j), ad, bd, id_s, kk > 0 ? 1u : 0u);
    }
    tc::mma_commit(bar_s(j));
  };
  // O(j) = P(j) V(j) into O buffer j&1 (bf16: hi part then lo part)
  auto issue_o = [&](int j) {
    tc::tc_fence_after();
    const uint32_t vb = smem_u32(vs + (j % kNBuf) * kKVBytes);
    const int parts = kBf16 ? 2 : 1;
    for (int part = 0; part < parts; ++part) {
      const uint32_t pa = smem_u32(part == 0 ? ph : pl);
#pragma unroll
      for (int kk = 0; kk < kBN / 16; ++kk) {
        const uint64_t ad = tc::smem_desc_sw128(pa + kk * 32, 16, 1024);
        const uint64_t bd = tc::smem_desc_sw128(vb + kk * 16 * 128, kBN * 128, 1024);
        tc::mma_f16(t_o(j), ad, bd, id_o, (part > 0 || kk > 0) ? 1u : 0u);
      }
    }
    tc::mma_commit(bar_o(j));
  };
  // acc = acc * alpha(j) + O(j)
  auto fold = [&](int j, float alpha) {
#pragma unroll
    for (int c0 = 0; c0 < kD; c0 += 32) {
      float o[32];
      tc::tmem_ld32(t_o(j) + lane_base + c0, o);
#pragma unroll
      for (int i = 0; i < 32; ++i) acc[c0 + i] = acc[c0 + i] * alpha + o[i];
    }
  };

  if (n_tiles > 0) {
    cp_async_wait<kNBuf - 2>();  // tile 0 resident
    tc::fence_proxy_async_smem();
    __syncthreads();
    if (tid == 0) issue_s(0);
  }

  for (int it = 0; it < n_tiles; ++it) {
    // [A] tile it+1 resident -> S(it+1) can start while this tile's softmax runs
    cp_async_wait<kNBuf - 3>();
    tc::fence_proxy_async_smem();
    tc::tc_fence_before();
    __syncthreads();
    if (tid == 0 && it + 1 < n_tiles) issue_s(it + 1);

    const bool ok_s = tc::mbar_wait(bar_s(it), (it >> 1) & 1);
    if (__syncthreads_or(!ok_s)) {
      failed = true;
      break;
    }
    tc::tc_fence_after();
    float s[kBN];
    tc::tmem_ld32(t_s(it) + lane_base, s);
    tc::tmem_ld32(t_s(it) + lane_base + 32, s + 32);
    const int tbase = it * kBN;
    float mx = -INFINITY;
#pragma unroll
    for (int c = 0; c < kBN; ++c) {
      s[c] = (tbase + c <= lim) ? s[c] * p.scale_log2 : -INFINITY;
      mx = fmaxf(mx, s[c]);
    }
    const float m_new = fmaxf(m_run, mx);
    const float m_use = m_new == -INFINITY ? 0.f : m_new;
    const float alpha = fast_exp2(m_run - m_use);
    m_run = m_new;

    // O(it-1) done: fold it, free its K/V buffer for tile it+3 and the P buffer
    if (it > 0) {
      const bool ok_o = tc::mbar_wait(bar_o(it - 1), ((it - 1) >> 1) & 1);
      if (__syncthreads_or(!ok_o)) {
        failed = true;
        break;
      }
      tc::tc_fence_after();
      fold(it - 1, alpha_prev);
    }
    if (it + kNBuf - 1 < n_tiles) load_kv(it + kNBuf - 1, (it + kNBuf - 1) % kNBuf);
    cp_async_commit();

    float sum = 0.f;
#pragma unroll
    for (int c = 0; c < kBN; c += 8) {
      uint32_t hi[4], lo[4];
#pragma unroll
      for (int e = 0; e < 8; e += 2) {
        const float a = fast_exp2(s[c + e] - m_use), bb = fast_exp2(s[c + e + 1] - m_use);
        sum += a + bb;
        split2<T>(a, bb, hi[e >> 1], lo[e >> 1]);
      }
      const uint32_t off = sw_off(row, c >> 3);
      *reinterpret_cast<uint4*>(ph + off) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
      if (kBf16) *reinterpret_cast<uint4*>(pl + off) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
    }
    l_run = l_run * alpha + sum;
    alpha_prev = alpha;
    tc::fence_proxy_async_smem();  // P stores -> visible to the tensor core
    tc::tc_fence_before();
    __syncthreads();  // [B]
    if (tid == 0) issue_o(it);
  }
  if (!failed && n_tiles > 0) {
    const int last = n_tiles - 1;
    const bool ok_o = tc::mbar_wait(bar_o(last), (last >> 1) & 1);
    if (__syncthreads_or(!ok_o)) {
      failed = true;
    } else {
      tc::tc_fence_after();
      fold(last, alpha_prev);
    }
  }
  cp_async_wait<0>();

  // ---- epilogue ----
  if (tok < nq) {
    const float inv = (l_run > 0.f && !failed) ? 1.f / l_run : 0.f;
    T* dst = reinterpret_cast<T*>(p.out) + (static_cast<int64_t>(q0 + tok) * p.Hq + hkv * p.n_rep + row % p.n_rep) * kD;
#pragma unroll
    for (int c = 0; c < kD; c += 8) {
      uint4 v;
      if (failed) {
        const float nan = __int_as_float(0x7fc00000);
        v = make_uint4(pack2<T>(nan, nan), pack2<T>(nan, nan), pack2<T>(nan, nan), pack2<T>(nan, nan));
      } else {
        v = make_uint4(pack2<T>(acc[c] * inv, acc[c + 1] * inv), pack2<T>(acc[c + 2] * inv, acc[c + 3] * inv),
                       pack2<T>(acc[c + 4] * inv, acc[c + 5] * inv), pack2<T>(acc[c + 6] * inv, acc[c + 7] * inv));
      }
      *reinterpret_cast<uint4*>(dst + c) = v;
    }
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace

// Launches the tcgen05 kernel; returns BPKV_ERR_UNSUPPORTED when the shape is
// not one it handles (head_dim 128, bf16/fp16, n_rep dividing 128).
int prefill_tc_launch(PrefillTcParams& p, int head_dim, int dtype, int max_seqlen_q, bool paged, cudaStream_t st) {
  if (head_dim != kD || (dtype != BPKV_BF16 && dtype != BPKV_F16) || kBM % p.n_rep != 0) return BPKV_ERR_UNSUPPORTED;
  const int TQ = kBM / p.n_rep;
  p.tiles_per_req = (max_seqlen_q + TQ - 1) / TQ;
  if (p.tiles_per_req == 0 || p.B == 0) return BPKV_OK;
  dim3 grid(p.B * p.tiles_per_req, p.Hkv);
  static bool raised[4][64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  const int variant = (dtype == BPKV_BF16 ? 0 : 2) + (paged ? 1 : 0);
#define BPKV_TC_LAUNCH(TY, PG)                                                                             \
  do {                                                                                                     \
    auto kern = prefill_tc_kernel<TY, PG>;                                                                 \
    if (dev < 64 && !raised[variant][dev]) {                                                               \
      if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes) != cudaSuccess) { \
        set_error("prefill_tc_launch:smem_attr");                                                          \
        return BPKV_ERR_CUDA;                                                                              \
      }                                                                                                    \
      raised[variant][dev] = true;                                                                         \
    }                                                                                                      \
    kern<<<grid, 128, kSmemBytes, st>>>(p);                                                                \
  } while (0)
  if (dtype == BPKV_BF16) {
    if (paged) BPKV_TC_LAUNCH(__nv_bfloat16, true); else BPKV_TC_LAUNCH(__nv_bfloat16, false);
  } else {
    if (paged) BPKV_TC_LAUNCH(__half, true); else BPKV_TC_LAUNCH(__half, false);
  }
#undef BPKV_TC_LAUNCH
  BPKV_RETURN_LAUNCH("prefill_tc_launch");
}

}  // namespace bpkv
