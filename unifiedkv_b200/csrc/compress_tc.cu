// Tensor-core (tcgen05 / TMEM) versions of the two scoring passes of the
// block-aligned SnapKV compression, sm_100a, head_dim 128, bf16 / fp16.
// Same math and outputs as the mma.sync passes in compress.cu:
//   pass 1 (stats):  S = Q_g K^T with the window rows of KV group g as M
//                    (up to two M-tiles of 128 rows), K tiles of 128 tokens as
//                    N; thread = row, so the running (max, sum-exp) of a row
//                    over the CTA's token range is thread-local;
//   pass 2 (scores): S^T = K Q_g^T, transposed on purpose: M = 128 tokens,
//                    N = the group's window rows (<= 256); two threads per
//                    token (half of the heads each), so p = exp(s - m_row) /
//                    l_row, the mean over each head's window rows and the max
//                    over the heads are thread-local up to one exchange ->
//                    headmax[g][token].
// Each CTA holds its group's Q in shared memory and streams a contiguous range
// of K tiles (about one CTA per SM): a load warp brings them by TMA (3-D tensor
// map over K, 128-byte swizzle, zero fill past the mid tokens) into a 3-deep
// ring, one thread issues the MMAs into double-buffered TMEM accumulators, and
// 8 warps evaluate the exponentials of tile j while the tensor core computes
// tile j+1.  1 in 8 exponentials is evaluated by a polynomial on the FMA pipe.
// Every wait is bounded.  No TMA multicast is used.
#include <cuda.h>

#include "common.cuh"
#include "score_tc.cuh"
#include "f32x2.cuh"
#include "tcgen05.cuh"

namespace bpkv {

namespace {

constexpr int kD = 128, kDB = 2, kTok = 128;   // head_dim, 64-col blocks, tokens per K tile
constexpr int kRowsMax = 256;                  // window rows of one KV group
constexpr int kQBytes = kDB * kRowsMax * 128;  // 64 KB
constexpr int kKBytes = kDB * kTok * 128;      // 32 KB per K tile
constexpr int kNK = 3;                         // K ring depth
constexpr int kComputeWarps = 16;
constexpr int kLoadWarp = kComputeWarps, kMmaWarp = kComputeWarps + 1;
constexpr int kThreads = (kComputeWarps + 2) * 32;
constexpr int kSmem = kQBytes + kNK * kKBytes + 1024 /*align*/ + 256 /*barriers*/ +
                      2 * kRowsMax * 2 * 4 /*pass 1: (m, l) merge of the row halves; pass 2: row offsets*/;
// every kEmu1-th / kEmu2-th exponential pair of pass 1 / pass 2 goes to the FMA pipe
constexpr int kEmu1 = 8, kEmu2 = 8;

struct __align__(64) ScoreTcArgs {
  CUtensorMap tmap_k;  // (d, token, kv head) over K, box (64, 128, 1), 128-B swizzle
  ScoreTcParams p;
};

__device__ __forceinline__ uint32_t sw_off(int row, int chunk) {
  return static_cast<uint32_t>(row * 128 + ((chunk ^ (row & 7)) << 4));
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, int c0, int c1, int c2,
                                            uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
      "[%5];\n" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(bar)
      : "memory");
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

// exp2 of 32 values x = s * scale + offs[c] (pre-negated per-value offsets, 8-byte aligned) or
// x = s * scale - off (one scalar), summed into a packed pair of partial sums
template <bool kPerValueOff, int kEmu>
__device__ __forceinline__ uint64_t exp2_sum32(const float* s, float scale, const float* offs, float off,
                                               uint64_t acc) {
  const uint64_t sc2 = pk2(scale, scale);
#pragma unroll
  for (int c = 0; c < 32; c += 2) {
    const uint64_t o2 = kPerValueOff ? *reinterpret_cast<const uint64_t*>(offs + c) : pk2(-off, -off);
    const uint64_t x2 = fma2(pk2(s[c], s[c + 1]), sc2, o2);
    uint64_t e2;
    if ((c >> 1) % kEmu == kEmu - 1) {
      e2 = exp2_poly2(x2);
    } else {
      float xa, xb;
      up2(x2, xa, xb);
      e2 = pk2(fast_exp2(xa), fast_exp2(xb));
    }
    acc = add2(acc, e2);
  }
  return acc;
}

// PASS 1: per (window row, token range) running (max, sum-exp) -> ml_part[row][chunk]
// PASS 2: per token, the max over the group's heads of the mean softmax mass -> headmax
template <typename T, int PASS>
__global__ void __launch_bounds__(kThreads, 1) score_tc_kernel(const __grid_constant__ ScoreTcArgs args) {
  const ScoreTcParams& p = args.p;
  pdl_wait();
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* qs = smem;
  uint8_t* ks = qs + kQBytes;  // kNK buffers
  uint64_t* bars = reinterpret_cast<uint64_t*>(ks + kNK * kKBytes);
  // bars: k_full[kNK], k_free[kNK], s_full[2], s_free[2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * kNK + 4);
  float* s_off = reinterpret_cast<float*>(bars + 32);   // PASS 1: [2][kRowsMax] (m, l) merge; PASS 2: per row -(m + log2 l)
  const int g = blockIdx.y, chunk = blockIdx.x;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int rows = p.n_rep * p.Wp;
  const int mtiles = (rows + 127) / 128;
  const int ntiles_all = (p.Tm + kTok - 1) / kTok;
  const int tile0 = chunk * p.tiles_per_chunk;
  const int ntiles = max(0, min(p.tiles_per_chunk, ntiles_all - tile0));
  // token tile of step j: pass 2 walks its range backwards, so it starts on the tiles that
  // pass 1 read last (still in L2: K_mid at 32K tokens is about the size of one die's L2,
  // and a forward walk would evict each tile just before it is needed)
  auto tile_of = [&](int j) { return PASS == 2 ? tile0 + ntiles - 1 - j : tile0 + j; };
  auto k_full = [&](int j) { return smem_u32(&bars[j % kNK]); };
  auto k_free = [&](int j) { return smem_u32(&bars[kNK + j % kNK]); };
  auto s_full = [&](int j) { return smem_u32(&bars[2 * kNK + (j & 1)]); };
  auto s_free = [&](int j) { return smem_u32(&bars[2 * kNK + 2 + (j & 1)]); };

  if (warp == 0) {
    tc::tmem_alloc(smem_u32(tmem_slot), 512);
    tc::tmem_relinquish();
  }
  if (tid == 0) {
    for (int i = 0; i < kNK; ++i) {
      tc::mbar_init(k_full(i), 1);
      tc::mbar_init(k_free(i), 1);
    }
    for (int i = 0; i < 2; ++i) {
      tc::mbar_init(s_full(i), 1);
      tc::mbar_init(s_free(i), kComputeWarps);
    }
    tc::fence_mbar_init();
  }
  load_q<T>(p, qs, g, PASS == 1 ? mtiles * 128 : rows, kThreads);
  cp_async_commit();
  if constexpr (PASS == 2) {
    // merge pass 1's partial (m, l) of this group's window rows over the token ranges
    // (fixed order) -> -(m + log2 l) per row, -inf for padding rows
    for (int r = tid; r < rows; r += kThreads) {
      if ((r % p.Wp) >= p.W) {
        s_off[r] = -INFINITY;
        continue;
      }
      const float2* src = p.ml_part + (static_cast<int64_t>(g) * rows + r) * p.n_chunks;
      float m = -INFINITY;
      for (int c = 0; c < p.n_chunks; ++c) m = fmaxf(m, src[c].x);
      float l = 0.f;
      for (int c = 0; c < p.n_chunks; ++c) l += src[c].y * exp2f(src[c].x - m);
      s_off[r] = -(m + log2f(l));
    }
  }
  cp_async_wait<0>();
  tc::fence_proxy_async_smem();
  tc::tc_fence_before();
  __syncthreads();  // Q staged, barriers initialised, TMEM address published
  tc::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  constexpr bool kBf16 = SplitP<T>::value;
  bool failed = false;

  if (warp == kLoadWarp) {
    // ---- K tiles by TMA: two 64-column boxes of 128 tokens (zero fill past the mid tokens) ----
    for (int j = 0; j < ntiles && !failed; ++j) {
      if (j >= kNK) failed = !tc::mbar_wait(k_free(j - kNK), ((j - kNK) / kNK) & 1);
      if (!failed && lane == 0) {
        const uint32_t bar = k_full(j);
        mbar_expect_tx(bar, kKBytes);
        uint8_t* dst = ks + (j % kNK) * kKBytes;
        const int t0 = p.sink + tile_of(j) * kTok;
        tma_load_3d(smem_u32(dst), &args.tmap_k, 0, t0, g, bar);
        tma_load_3d(smem_u32(dst + kTok * 128), &args.tmap_k, 64, t0, g, bar);
      }
      __syncwarp();
    }
  } else if (warp == kMmaWarp) {
    // ---- one thread issues the MMAs of tile j into TMEM buffer j & 1 ----
    const uint32_t qa = smem_u32(qs);
    for (int j = 0; j < ntiles && !failed; ++j) {
      failed = !tc::mbar_wait(k_full(j), (j / kNK) & 1);
      if (!failed && j >= 2) failed = !tc::mbar_wait(s_free(j), ((j - 2) >> 1) & 1);
      if (!failed && lane == 0) {
        tc::tc_fence_after();
        const uint32_t kb = smem_u32(ks + (j % kNK) * kKBytes);
        const uint32_t dbuf = tmem + static_cast<uint32_t>((j & 1) * 256);
        if constexpr (PASS == 1) {
          const uint32_t idesc = tc::idesc_f16(kBf16, false, false, 128, kTok);
          for (int t = 0; t < mtiles; ++t) {
#pragma unroll
            for (int kk = 0; kk < kD / 16; ++kk) {
              const uint32_t koff = (kk & 3) * 32;
              const uint64_t ad = tc::smem_desc_sw128(qa + (kk >> 2) * (kRowsMax * 128) + t * 128 * 128 + koff, 16, 1024);
              const uint64_t bd = tc::smem_desc_sw128(kb + (kk >> 2) * (kTok * 128) + koff, 16, 1024);
              tc::mma_f16(dbuf + t * 128, ad, bd, idesc, kk > 0 ? 1u : 0u);
            }
          }
        } else {
          const uint32_t idesc = tc::idesc_f16(kBf16, false, false, 128, rows);
#pragma unroll
          for (int kk = 0; kk < kD / 16; ++kk) {
            const uint32_t koff = (kk & 3) * 32;
            const uint64_t ad = tc::smem_desc_sw128(kb + (kk >> 2) * (kTok * 128) + koff, 16, 1024);
            const uint64_t bd = tc::smem_desc_sw128(qa + (kk >> 2) * (kRowsMax * 128) + koff, 16, 1024);
            tc::mma_f16(dbuf, ad, bd, idesc, kk > 0 ? 1u : 0u);
          }
        }
        tc::mma_commit(s_full(j));
        tc::mma_commit(k_free(j));
      }
      __syncwarp();
    }
  } else {
    // ---- compute warps ----
    auto wait = [&](uint32_t bar, uint32_t parity) {
      if (failed) return;
      const bool r = tc::mbar_wait(bar, parity);
      if (!__all_sync(0xffffffffu, r)) failed = true;
    };
    auto release = [&](int j) {  // this warp is done reading TMEM buffer j & 1
      tc::tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(s_free(j));
    };
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    if constexpr (PASS == 1) {
      // warp w: TMEM lane quarter w % 4, M-tile (w / 4) % 2, column half w / 8 of each K tile
      const int mt = (warp >> 2) & 1, ch = warp >> 3;
      const int row = mt * 128 + (warp & 3) * 32 + lane;
      float m_ref = -INFINITY, l = 0.f;  // this half-row: sum of exp2(x - m_ref)
      for (int j = 0; j < ntiles; ++j) {
        wait(s_full(j), (j >> 1) & 1);
        tc::tc_fence_after();
        if (mt < mtiles && !failed) {
          const uint32_t tcol = tmem + static_cast<uint32_t>((j & 1) * 256 + mt * 128 + ch * 64) + lane_base;
          const int nvalid = min(kTok, p.Tm - tile_of(j) * kTok) - ch * 64;  // valid columns of this half
          auto load = [&](int c0, float* a) {
            tc::tmem_ld32(tcol + c0, a);
            if (c0 + 32 > nvalid) {
#pragma unroll
              for (int c = 0; c < 32; ++c) a[c] = c0 + c < nvalid ? a[c] : -INFINITY;
            }
          };
          auto tile_sum = [&](float ref, float& mx) {  // sum of exp2(s*scale - ref) and the raw max
            uint64_t acc = 0ull;
            float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
            for (int c0 = 0; c0 < 64; c0 += 32) {
              float a[32];
              load(c0, a);
#pragma unroll
              for (int c = 0; c < 32; ++c) m4[c & 3] = fmaxf(m4[c & 3], a[c]);
              acc = exp2_sum32<false, kEmu1>(a, p.scale_log2, nullptr, ref, acc);
            }
            mx = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3]));
            float sa, sb;
            up2(acc, sa, sb);
            return sa + sb;
          };
          // tcgen05.ld is warp-collective: every TMEM load below is executed by the whole
          // warp (branches on __any_sync), each lane keeping or dropping the result by its
          // own row's condition
          const bool no_ref = m_ref == -INFINITY;
          if (__any_sync(0xffffffffu, no_ref)) {  // no reference yet: take this tile's max first
            float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
            for (int c0 = 0; c0 < 64; c0 += 32) {
              float a[32];
              load(c0, a);
#pragma unroll
              for (int c = 0; c < 32; ++c) m4[c & 3] = fmaxf(m4[c & 3], a[c]);
            }
            if (no_ref) m_ref = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3])) * p.scale_log2;  // scale > 0
          }
          // one pass with the current (lazily moved) reference; the tile's max comes out of it.
          // A row still without a reference has only -inf scores: its terms are 0 for any ref.
          const bool has_ref = m_ref != -INFINITY;
          float mx;
          float sum = tile_sum(has_ref ? m_ref : 0.f, mx);
          const float mxs = mx * p.scale_log2;
          const bool moved = has_ref && mxs > m_ref + 8.f;
          const bool redo = moved && mxs > m_ref + 120.f;  // terms may have overflowed
          if (__any_sync(0xffffffffu, redo)) {
            float mx2;
            const float sum2 = tile_sum(redo ? mxs : (has_ref ? m_ref : 0.f), mx2);
            if (redo) sum = sum2;
          }
          if (moved) {
            if (!redo) sum *= fast_exp2(m_ref - mxs);
            l = l * fast_exp2(m_ref - mxs) + sum;
            m_ref = mxs;
          } else if (has_ref) {
            l += sum;
          }
        }
        release(j);
      }
      // merge the two column halves of each row
      float* ml_s = s_off;  // [2 halves][kRowsMax][m, l] (the pass-2 areas, unused here)
      if (mt < mtiles) {
        ml_s[(ch * kRowsMax + row) * 2] = m_ref;
        ml_s[(ch * kRowsMax + row) * 2 + 1] = l;
      }
      asm volatile("bar.sync 1, %0;\n" ::"n"(32 * kComputeWarps) : "memory");
      if (ch == 0 && mt < mtiles && row < rows) {
        const float m1 = ml_s[(kRowsMax + row) * 2], l1 = ml_s[(kRowsMax + row) * 2 + 1];
        const float M = fmaxf(m_ref, m1);
        const float L = M == -INFINITY ? 0.f
                                       : (m_ref == -INFINITY ? 0.f : l * fast_exp2(m_ref - M)) +
                                             (m1 == -INFINITY ? 0.f : l1 * fast_exp2(m1 - M));
        const int grow = g * p.n_rep * p.Wp + row;
        p.ml_part[static_cast<int64_t>(grow) * p.n_chunks + chunk] =
            failed ? make_float2(__int_as_float(0x7fc00000), 0.f) : make_float2(M, L);
      }
    } else {
      // warp w: TMEM lane quarter w % 4 (its 32 tokens), head slot hs = w / 4: heads hs, hs + 4, ...
      const int hs = warp >> 2;
      const int tt = (warp & 3) * 32 + lane;
      const float invW = 1.f / static_cast<float>(p.W);
      for (int j = 0; j < ntiles; ++j) {
        wait(s_full(j), (j >> 1) & 1);
        tc::tc_fence_after();
        float best = -INFINITY;
        if (!failed) {
          const uint32_t base = tmem + static_cast<uint32_t>((j & 1) * 256) + lane_base;
          for (int r = hs; r < p.n_rep; r += 4) {  // head r: window columns r*Wp .. r*Wp+Wp-1
            uint64_t acc = 0ull;
            for (int i0 = 0; i0 < p.Wp; i0 += 32) {
              const int c0 = r * p.Wp + i0;
              float a[32];
              if (i0 + 32 <= p.Wp) {
                tc::tmem_ld32(base + c0, a);
              } else {  // a 16-column remainder (Wp is a multiple of 16)
                tc::tmem_ld16(base + c0, a);
#pragma unroll
                for (int c = 16; c < 32; ++c) a[c] = -INFINITY;
              }
              acc = exp2_sum32<true, kEmu2>(a, p.scale_log2, s_off + c0, 0.f, acc);
            }
            float sa, sb;
            up2(acc, sa, sb);
            best = fmaxf(best, (sa + sb) * invW);
          }
        }
        release(j);
        // each head slot writes its own row; the max over the slots is taken by the block reduction
        const int t = tile_of(j) * kTok + tt;
        if (hs < p.hm_slots && t < p.Tm)
          p.headmax[static_cast<int64_t>(g * p.hm_slots + hs) * p.Tm + t] = failed ? __int_as_float(0x7fc00000) : best;
      }
    }
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, 512);
  }
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no libcuda link).
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  }
  return fn;
}

}  // namespace

int score_tc_pass(ScoreTcParams& p, int head_dim, int dtype, int pass, cudaStream_t st) {
  const int rows = p.n_rep * p.Wp;
  if (head_dim != kD || rows > kRowsMax || (dtype != BPKV_BF16 && dtype != BPKV_F16)) return BPKV_ERR_UNSUPPORTED;
  if ((p.k_st * 2) % 16 != 0 || (p.k_sh * 2) % 16 != 0) return BPKV_ERR_UNSUPPORTED;
  EncodeTiledFn enc = encode_fn();
  if (enc == nullptr) return BPKV_ERR_UNSUPPORTED;
  const int ntiles = (p.Tm + kTok - 1) / kTok;
  p.hm_slots = min(4, p.n_rep);  // pass 2's head slots (headmax rows per KV group)
  if (pass == 1) {
    // about one CTA per SM: split each group's tiles into contiguous ranges (p.n_chunks
    // arrives as the workspace's capacity of partial-stat slots per row)
    int n = max(1, min(min(p.n_chunks, ntiles), sm_count() / max(1, p.Hkv)));
    p.tiles_per_chunk = (ntiles + n - 1) / n;
    p.n_chunks = (ntiles + p.tiles_per_chunk - 1) / p.tiles_per_chunk;
  }
  ScoreTcArgs args;
  memset(&args, 0, sizeof(args));
  args.p = p;
  {
    // K viewed as (d, token, kv head): tokens past sink + Lm read as zero
    const cuuint64_t dims[3] = {static_cast<cuuint64_t>(kD), static_cast<cuuint64_t>(p.sink + p.Lm),
                                static_cast<cuuint64_t>(p.Hkv)};
    const cuuint64_t strides[2] = {static_cast<cuuint64_t>(p.k_st) * 2, static_cast<cuuint64_t>(p.k_sh) * 2};
    const cuuint32_t box[3] = {64, kTok, 1};
    const cuuint32_t estr[3] = {1, 1, 1};
    if (enc(&args.tmap_k, dtype == BPKV_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3,
            const_cast<void*>(p.k), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS) {
      set_error("block_score_tc:tensor_map_encode_failed");
      return BPKV_ERR_CUDA;
    }
  }
  static bool raised[4][64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  const int v = (dtype == BPKV_BF16 ? 0 : 2) + (pass == 1 ? 0 : 1);
  dim3 grid(p.n_chunks, p.Hkv);
#define BPKV_SCORE_TC(TY, PS)                                                                   \
  do {                                                                                          \
    auto kern = score_tc_kernel<TY, PS>;                                                        \
    if (dev < 64 && !raised[v][dev]) {                                                          \
      if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem) != cudaSuccess) { \
        set_error("block_score_tc:smem_attr");                                                  \
        return BPKV_ERR_CUDA;                                                                   \
      }                                                                                         \
      raised[v][dev] = true;                                                                    \
    }                                                                                           \
    if (launch_pdl(kern, grid, dim3(kThreads), kSmem, st, args) != cudaSuccess) {             \
      set_error("block_score_tc_launch:launch");                                                \
      return BPKV_ERR_CUDA;                                                                     \
    }                                                                                           \
  } while (0)
  if (dtype == BPKV_BF16) {
    if (pass == 1) BPKV_SCORE_TC(__nv_bfloat16, 1); else BPKV_SCORE_TC(__nv_bfloat16, 2);
  } else {
    if (pass == 1) BPKV_SCORE_TC(__half, 1); else BPKV_SCORE_TC(__half, 2);
  }
#undef BPKV_SCORE_TC
  BPKV_RETURN_LAUNCH("block_score_tc_launch");
}

}  // namespace bpkv
