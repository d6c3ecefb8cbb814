// Tensor-core (tcgen05 / TMEM) versions of the two scoring passes of the
// block-aligned SnapKV compression, sm_100a, head_dim 128, bf16 / fp16.
// Same math and outputs as the mma.sync passes in compress.cu:
//   pass 1 (stats):  S = Q_g K^T with the window rows of KV group g as M
//                    (two M-tiles of 128 rows, padded), K tiles of 128 tokens
//                    as N; thread = row, so the running (max, sum-exp) of a row
//                    over the CTA's token chunk is thread-local;
//   pass 2 (scores): S^T = K Q_g^T, transposed on purpose: M = 128 tokens,
//                    N = the group's window rows (<= 256); thread = token, so
//                    p = exp(s - m_row) / l_row, the mean over each head's
//                    window rows and the max over the group's heads are all
//                    thread-local -> headmax[g][token].
// K tiles are gathered with 16-byte cp.async into the 128-byte-swizzled UMMA
// layout and arrive on an mbarrier; MMAs are issued by one thread and
// committed to an mbarrier; every wait is bounded.
#include "common.cuh"
#include "tcgen05.cuh"

namespace bpkv {

struct ScoreTcParams {
  const void* k;
  const void* q;
  int Hkv, n_rep, W, Wp, Lm, Tm, sink, n_chunks;
  int64_t k_sh, k_st, q_sh, q_st;
  float scale_log2;
  float2* ml_part;  // [Hq*Wp][n_chunks]
  const float2* ml; // [Hq*Wp]
  float* headmax;   // [Hkv][Tm]
};

namespace {

constexpr int kD = 128, kDB = 2, kTok = 128;   // head_dim, 64-col blocks, tokens per K tile
constexpr int kRowsMax = 256;                  // window rows of one KV group
constexpr int kQBytes = kDB * kRowsMax * 128;  // 64 KB
constexpr int kKBytes = kDB * kTok * 128;      // 32 KB per K tile
constexpr int kStatTiles = 8;                  // pass 1: 1024 tokens per CTA
constexpr int kSmem1 = kQBytes + 2 * kKBytes + 1024 + 64;
constexpr int kSmem2 = kQBytes + kKBytes + 1024 + 64 + kRowsMax * 4;

__device__ __forceinline__ uint32_t sw_off(int row, int chunk) {
  return static_cast<uint32_t>(row * 128 + ((chunk ^ (row & 7)) << 4));
}
__device__ __forceinline__ void cp_async_arrive(uint32_t bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];\n" ::"r"(bar) : "memory");
}

// Q rows of group g (row = r*Wp + i, zero for i >= W or row >= rows) -> [db][row][128 B]
template <typename T>
__device__ void load_q(const ScoreTcParams& p, uint8_t* qs, int g, int rows_pad, int nthr) {
  const T* qg = reinterpret_cast<const T*>(p.q);
  const int rows = p.n_rep * p.Wp;
  for (int ci = threadIdx.x; ci < rows_pad * 16; ci += nthr) {
    const int row = ci / 16, ch = ci % 16;
    const int r = row / p.Wp, i = row % p.Wp;
    const bool ok = row < rows && i < p.W;
    const T* src = qg + static_cast<int64_t>(g * p.n_rep + r) * p.q_sh + static_cast<int64_t>(i) * p.q_st + ch * 8;
    cp_async16(smem_u32(qs + (ch >> 3) * (kRowsMax * 128) + sw_off(row, ch & 7)), ok ? (const void*)src : (const void*)qg,
               ok);
  }
}

// K tile (mid tokens t0 .. t0+127, zero past Lm) -> [db][token][128 B]
template <typename T>
__device__ void load_k(const ScoreTcParams& p, uint8_t* kb, int g, int t0, int nthr) {
  const T* kg = reinterpret_cast<const T*>(p.k);
  for (int ci = threadIdx.x; ci < kTok * 16; ci += nthr) {
    const int tt = ci / 16, ch = ci % 16;
    const int t = t0 + tt;
    const bool ok = t < p.Lm;
    const T* src = kg + static_cast<int64_t>(g) * p.k_sh + static_cast<int64_t>(p.sink + t) * p.k_st + ch * 8;
    cp_async16(smem_u32(kb + (ch >> 3) * (kTok * 128) + sw_off(tt, ch & 7)), ok ? (const void*)src : (const void*)kg, ok);
  }
}

// ---- pass 1: per (window row, 1024-token chunk) running max / sum-exp ----
template <typename T>
__global__ void __launch_bounds__(256, 1) score_stats_tc_kernel(ScoreTcParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* qs = smem;
  uint8_t* ks = qs + kQBytes;  // 2 buffers
  uint64_t* bars = reinterpret_cast<uint64_t*>(ks + 2 * kKBytes);  // k0, k1, s
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 3);
  const int g = blockIdx.y, chunk = blockIdx.x;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int rows = p.n_rep * p.Wp;
  const int mtiles = (rows + 127) / 128;
  const int tile0 = chunk * kStatTiles;
  const int ntiles = min(kStatTiles, (p.Tm + kTok - 1) / kTok - tile0);

  if (warp == 0) {
    tc::tmem_alloc(smem_u32(tmem_slot), 256);
    tc::tmem_relinquish();
  }
  if (tid == 0) {
    tc::mbar_init(smem_u32(&bars[0]), 256);
    tc::mbar_init(smem_u32(&bars[1]), 256);
    tc::mbar_init(smem_u32(&bars[2]), 1);
    tc::fence_mbar_init();
  }
  load_q<T>(p, qs, g, mtiles * 128, 256);
  cp_async_commit();
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  load_k<T>(p, ks, g, tile0 * kTok, 256);
  cp_async_arrive(smem_u32(&bars[0]));
  cp_async_wait<0>();  // Q

  constexpr bool kBf16 = SplitP<T>::value;
  const uint32_t idesc = tc::idesc_f16(kBf16, false, false, 128, kTok);
  const int mt = warp >> 2;                      // this warp's M-tile
  const int row = mt * 128 + (warp & 3) * 32 + lane;
  const uint32_t tcol = tmem + static_cast<uint32_t>(mt * 128) + (static_cast<uint32_t>((warp & 3) * 32) << 16);
  float m = -INFINITY, l = 0.f;
  bool failed = false;
  for (int j = 0; j < ntiles; ++j) {
    if (j + 1 < ntiles) {
      load_k<T>(p, ks + ((j + 1) & 1) * kKBytes, g, (tile0 + j + 1) * kTok, 256);
      cp_async_arrive(smem_u32(&bars[(j + 1) & 1]));
    }
    bool ok = tc::mbar_wait(smem_u32(&bars[j & 1]), (j >> 1) & 1);
    tc::fence_proxy_async_smem();
    if (__syncthreads_or(!ok)) {
      failed = true;
      break;
    }
    if (tid == 0) {
      tc::tc_fence_after();
      const uint32_t qa = smem_u32(qs), kb = smem_u32(ks + (j & 1) * kKBytes);
      for (int t = 0; t < mtiles; ++t) {
#pragma unroll
        for (int kk = 0; kk < kD / 16; ++kk) {
          const uint32_t koff = (kk & 3) * 32;
          const uint64_t ad = tc::smem_desc_sw128(qa + (kk >> 2) * (kRowsMax * 128) + t * 128 * 128 + koff, 16, 1024);
          const uint64_t bd = tc::smem_desc_sw128(kb + (kk >> 2) * (kTok * 128) + koff, 16, 1024);
          tc::mma_f16(tmem + t * 128, ad, bd, idesc, kk > 0 ? 1u : 0u);
        }
      }
      tc::mma_commit(smem_u32(&bars[2]));
    }
    ok = tc::mbar_wait(smem_u32(&bars[2]), j & 1);
    if (__syncthreads_or(!ok)) {
      failed = true;
      break;
    }
    tc::tc_fence_after();
    if (mt < mtiles) {
      const int tb = (tile0 + j) * kTok;
      float sv[kTok];
#pragma unroll
      for (int c0 = 0; c0 < kTok; c0 += 32) tc::tmem_ld32(tcol + c0, sv + c0);
      // scale > 0: the max of the scaled row is the scaled max of the raw row.
      // Four independent max / sum chains; only the last tile needs the bound.
      const int nvalid = min(kTok, p.Tm - tb);
      if (nvalid < kTok) {
#pragma unroll
        for (int c = 0; c < kTok; ++c)
          if (c >= nvalid) sv[c] = -INFINITY;
      }
      float mx4[4] = {sv[0], sv[1], sv[2], sv[3]};
#pragma unroll
      for (int c = 4; c < kTok; ++c) mx4[c & 3] = fmaxf(mx4[c & 3], sv[c]);
      const float mx = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3]));
      const float mn = fmaxf(m, mx * p.scale_log2);
      float s4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int c = 0; c < kTok; ++c) s4[c & 3] += fast_exp2(fmaf(sv[c], p.scale_log2, -mn));
      const float sum = (s4[0] + s4[1]) + (s4[2] + s4[3]);
      l = l * fast_exp2(m - mn) + sum;
      m = mn;
    }
    tc::tc_fence_before();
    __syncthreads();  // S in TMEM and this K buffer are reused
  }
  cp_async_wait<0>();
  if (row < rows) {
    const int grow = g * p.n_rep * p.Wp + row;
    p.ml_part[static_cast<int64_t>(grow) * p.n_chunks + chunk] =
        failed ? make_float2(__int_as_float(0x7fc00000), 0.f) : make_float2(m, l);
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, 256);
  }
}

// ---- pass 2: per token, max over the group's heads of the mean softmax mass ----
template <typename T>
__global__ void __launch_bounds__(128, 2) score_tokens_tc_kernel(ScoreTcParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* qs = smem;
  uint8_t* kb = qs + kQBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(kb + kKBytes);  // k, s
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2);
  float* s_off = reinterpret_cast<float*>(bars + 8);  // per window row: m + log2(l), +inf if padding
  const int g = blockIdx.y, tile = blockIdx.x;
  const int tid = threadIdx.x, warp = tid >> 5;
  const int rows = p.n_rep * p.Wp;

  if (warp == 0) {
    tc::tmem_alloc(smem_u32(tmem_slot), 256);
    tc::tmem_relinquish();
  }
  if (tid == 0) {
    tc::mbar_init(smem_u32(&bars[0]), 128);
    tc::mbar_init(smem_u32(&bars[1]), 1);
    tc::fence_mbar_init();
  }
  load_q<T>(p, qs, g, rows, 128);
  cp_async_commit();
  for (int r = tid; r < rows; r += 128) {
    const float2 st = p.ml[static_cast<int64_t>(g) * p.n_rep * p.Wp + r];
    s_off[r] = (r % p.Wp) < p.W ? st.x + log2f(st.y) : INFINITY;
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  load_k<T>(p, kb, g, tile * kTok, 128);
  cp_async_arrive(smem_u32(&bars[0]));
  cp_async_wait<0>();
  bool ok = tc::mbar_wait(smem_u32(&bars[0]), 0);
  tc::fence_proxy_async_smem();
  bool failed = __syncthreads_or(!ok);
  if (!failed && tid == 0) {
    tc::tc_fence_after();
    constexpr bool kBf16 = SplitP<T>::value;
    const uint32_t idesc = tc::idesc_f16(kBf16, false, false, 128, rows);
    const uint32_t ka = smem_u32(kb), qa = smem_u32(qs);
#pragma unroll
    for (int kk = 0; kk < kD / 16; ++kk) {
      const uint32_t koff = (kk & 3) * 32;
      const uint64_t ad = tc::smem_desc_sw128(ka + (kk >> 2) * (kTok * 128) + koff, 16, 1024);
      const uint64_t bd = tc::smem_desc_sw128(qa + (kk >> 2) * (kRowsMax * 128) + koff, 16, 1024);
      tc::mma_f16(tmem, ad, bd, idesc, kk > 0 ? 1u : 0u);
    }
    tc::mma_commit(smem_u32(&bars[1]));
  }
  if (!failed) {
    ok = tc::mbar_wait(smem_u32(&bars[1]), 0);
    failed = __syncthreads_or(!ok);
  }
  const int t = tile * kTok + tid;
  if (!failed) {
    tc::tc_fence_after();
    const uint32_t base = tmem + (static_cast<uint32_t>(warp * 32) << 16);
    const float invW = 1.f / static_cast<float>(p.W);
    float best = -INFINITY;
    for (int r = 0; r < p.n_rep; ++r) {  // head r: window columns r*Wp .. r*Wp+Wp-1
      float cur = 0.f;
      for (int i0 = 0; i0 < p.Wp; i0 += 16) {
        const int c0 = r * p.Wp + i0;
        float sv[16];
        tc::tmem_ld16(base + c0, sv);
        float c4[4] = {0.f, 0.f, 0.f, 0.f};  // four independent chains, then a fixed-order add
#pragma unroll
        for (int i = 0; i < 16; ++i) c4[i & 3] += fast_exp2(fmaf(sv[i], p.scale_log2, -s_off[c0 + i]));
        cur += (c4[0] + c4[1]) + (c4[2] + c4[3]);
      }
      best = fmaxf(best, cur * invW);
    }
    if (t < p.Tm) p.headmax[static_cast<int64_t>(g) * p.Tm + t] = best;
  } else if (t < p.Tm) {
    p.headmax[static_cast<int64_t>(g) * p.Tm + t] = __int_as_float(0x7fc00000);
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, 256);
  }
}

}  // namespace

// Pass 1 + pass 2 on tcgen05 when the shape allows (head_dim 128, <= 256 window
// rows per KV group, bf16/fp16); BPKV_ERR_UNSUPPORTED otherwise.  Sets
// p.n_chunks (1024-token chunks) for the stats reduction that runs between.
int score_tc_pass(ScoreTcParams& p, int head_dim, int dtype, int pass, cudaStream_t st) {
  const int rows = p.n_rep * p.Wp;
  if (head_dim != kD || rows > kRowsMax || (dtype != BPKV_BF16 && dtype != BPKV_F16)) return BPKV_ERR_UNSUPPORTED;
  const int ntok_tiles = (p.Tm + kTok - 1) / kTok;
  static bool raised[4][64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  const int v = (dtype == BPKV_BF16 ? 0 : 2) + (pass == 1 ? 0 : 1);
  auto raise = [&](const void* fn, int bytes) {
    if (dev < 64 && !raised[v][dev]) {
      cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
      raised[v][dev] = true;
    }
  };
  if (pass == 1) {
    p.n_chunks = (ntok_tiles + kStatTiles - 1) / kStatTiles;
    dim3 grid(p.n_chunks, p.Hkv);
    if (dtype == BPKV_BF16) {
      raise(reinterpret_cast<const void*>(score_stats_tc_kernel<__nv_bfloat16>), kSmem1);
      score_stats_tc_kernel<__nv_bfloat16><<<grid, 256, kSmem1, st>>>(p);
    } else {
      raise(reinterpret_cast<const void*>(score_stats_tc_kernel<__half>), kSmem1);
      score_stats_tc_kernel<__half><<<grid, 256, kSmem1, st>>>(p);
    }
  } else {
    dim3 grid(ntok_tiles, p.Hkv);
    if (dtype == BPKV_BF16) {
      raise(reinterpret_cast<const void*>(score_tokens_tc_kernel<__nv_bfloat16>), kSmem2);
      score_tokens_tc_kernel<__nv_bfloat16><<<grid, 128, kSmem2, st>>>(p);
    } else {
      raise(reinterpret_cast<const void*>(score_tokens_tc_kernel<__half>), kSmem2);
      score_tokens_tc_kernel<__half><<<grid, 128, kSmem2, st>>>(p);
    }
  }
  BPKV_RETURN_LAUNCH("block_score_tc_launch");
}

}  // namespace bpkv
