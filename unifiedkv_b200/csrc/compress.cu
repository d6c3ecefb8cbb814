// Block-aligned SnapKV compression on sm_100a: observation-window block
// scoring, deterministic top-k block selection and compacting writeback into
// pool pages.
//
// Reference math (core/compress.py:100-144, core/scheduler.py:565-616):
//   K_mid = K[:, Ls : L-Lo] zero-padded to N*16 tokens,
//   A = softmax(Q_obs . repeat_kv(K_mid)^T * d^-1/2)   [h_q, W, N*16]
//   S = A.mean(queries).max(heads); block = S.view(N,16).sum(-1); max_pool1d(3,1,1)
//   top-k blocks, ascending.
// The reference materialises A (h_q*W*N*16 floats) and a repeat_kv copy of
// K_mid.  Here nothing of that size is written:
//   pass 1  score_tile_kernel<STATS>: per (window row, token chunk) online
//           max / sum-exp over the chunk, tensor-core QK^T (mma.m16n8k16).
//   reduce  stats_reduce_kernel: per row (m, l) over chunks, fixed order.
//   pass 2  score_tile_kernel<SCORE>: recomputes QK^T, p = exp(s - m)/l,
//           mean over the head's window rows, max over the group's n_rep heads
//           -> headmax[kv_head][token].
//   blocks  block_reduce_kernel: max over kv heads, 16-token sums, max-pool 3.
// Every reduction has a fixed order, so the scores are bit-reproducible run to
// run.  K is read twice (once per pass) straight from HBM in 16-byte cp.async
// copies; Q of a KV group stays in shared memory for the CTA's token chunk.
// For head_dim 128 (bf16 / fp16, window rows of a KV group within the tcgen05
// kernel's limit) both passes run instead as the tcgen05 kernels of
// compress_tc.cu, whose pass 2 merges the per-range row statistics itself (no
// reduce launch); the mma.sync kernels here serve the other shapes.  On the
// tcgen05 path every launch of a compression step (both passes, the block
// reduction, the top-k, the compaction) is a programmatic dependent launch of
// the one before it (launch_pdl), each kernel waiting for its predecessor
// first; the top-k and the compaction are launched that way on both paths.
#include <type_traits>

#include "common.cuh"
#include "score_tc.cuh"

namespace bpkv {

namespace {

constexpr int kTileTok = 64;    // tokens per mma tile
constexpr int kChunkTiles = 4;  // tiles per CTA -> 256 tokens per CTA
constexpr int kScoreWarps = 8;

struct ScoreParams {
  const void* k;
  const void* q;
  int Hkv, Hq, n_rep, L, W, Wp, D, sink, obs;
  int Lm;  // real mid tokens = L - sink - obs
  int Tm;  // padded mid tokens = 16 * N
  int n_chunks;
  int64_t k_sh, k_st, q_sh, q_st;
  float scale_log2;
  float2* ml_part;  // [Hq*Wp][n_chunks] (m in log2 units, l)
  float2* ml;       // [Hq*Wp]
  float* headmax;   // [Hkv][Tm]
};

template <typename T, int D, bool SCORE>
__global__ void __launch_bounds__(kScoreWarps * 32) score_tile_kernel(ScoreParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  constexpr int ROWB = D * 2;
  constexpr int CH = D / 8;
  constexpr int SWM = CH >= 8 ? 7 : CH - 1;  // XOR swizzle stays inside a row
  const int g = blockIdx.y;  // kv head
  const int chunk = blockIdx.x;
  const int rows = p.n_rep * p.Wp;  // padded window rows of this group
  const int R16 = rows / 16;
  uint8_t* qs = smem;
  uint8_t* ks = smem + static_cast<size_t>(rows) * ROWB;  // 2 K tiles
  float* cs = reinterpret_cast<float*>(ks + 2 * kTileTok * ROWB);  // [R16][64] (SCORE)
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const T* qg = reinterpret_cast<const T*>(p.q);
  const T* kg = reinterpret_cast<const T*>(p.k);

  // ---- load Q of the group (rows r*Wp + i, zero for i >= W) ----
  for (int ci = tid; ci < rows * CH; ci += blockDim.x) {
    const int row = ci / CH, ch = ci % CH;
    const int r = row / p.Wp, i = row % p.Wp;
    const bool ok = i < p.W;
    const T* src = qg + static_cast<int64_t>(g * p.n_rep + r) * p.q_sh + static_cast<int64_t>(i) * p.q_st + ch * 8;
    cp_async16(smem_u32(qs + row * ROWB + ((ch ^ (row & SWM)) << 4)), ok ? (const void*)src : (const void*)qg, ok);
  }
  const int tile0 = chunk * kChunkTiles;
  const int ntiles_total = (p.Tm + kTileTok - 1) / kTileTok;
  const int ntiles = min(kChunkTiles, ntiles_total - tile0);
  auto load_k = [&](int tile, int buf) {
    uint8_t* kb = ks + buf * kTileTok * ROWB;
    for (int ci = tid; ci < kTileTok * CH; ci += blockDim.x) {
      const int tok = ci / CH, ch = ci % CH;
      const int t = tile * kTileTok + tok;  // mid token index
      const bool ok = t < p.Lm;
      const T* src = kg + static_cast<int64_t>(g) * p.k_sh + static_cast<int64_t>(p.sink + t) * p.k_st + ch * 8;
      cp_async16(smem_u32(kb + tok * ROWB + ((ch ^ (tok & SWM)) << 4)), ok ? (const void*)src : (const void*)kg, ok);
    }
  };
  load_k(tile0, 0);
  cp_async_commit();

  // per-row running stats for STATS (rows owned by warp: rb = warp, warp+8, ...)
  float* m_s = cs;           // reuse: [rows]
  float* l_s = cs + rows;    // [rows]
  if (!SCORE) {
    for (int r = tid; r < rows; r += blockDim.x) {
      m_s[r] = -INFINITY;
      l_s[r] = 0.f;
    }
  }
  const int gq = lane >> 2, cq = lane & 3;

  for (int it = 0; it < ntiles; ++it) {
    if (it + 1 < ntiles) load_k(tile0 + it + 1, (it + 1) & 1);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    const uint32_t kb = smem_u32(ks + (it & 1) * kTileTok * ROWB);
    const uint32_t qb = smem_u32(qs);
    const int tbase = (tile0 + it) * kTileTok;
    for (int rb = warp; rb < R16; rb += kScoreWarps) {
      float acc[8][4];
#pragma unroll
      for (int n = 0; n < 8; ++n) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.f;
      const int mi = lane >> 3, rr = lane & 7;
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        uint32_t a[4];
        {
          const int row = rb * 16 + (mi & 1) * 8 + rr;
          const int ch = 2 * kk + (mi >> 1);
          ldmatrix_x4(qb + row * ROWB + ((ch ^ (row & SWM)) << 4), a[0], a[1], a[2], a[3]);
        }
#pragma unroll
        for (int np = 0; np < 4; ++np) {
          const int tok = np * 16 + rr + 8 * (mi >> 1);
          const int ch = 2 * kk + (mi & 1);
          uint32_t b0, b1, b2, b3;
          ldmatrix_x4(kb + tok * ROWB + ((ch ^ (tok & SWM)) << 4), b0, b1, b2, b3);
          mma16816<T>(acc[2 * np], a, b0, b1);
          mma16816<T>(acc[2 * np + 1], a, b2, b3);
        }
      }
      // lane holds rows (rb*16+gq) [acc[.][0..1]] and (+8) [acc[.][2..3]],
      // tokens n*8 + 2cq + {0,1}
      const int rowA = rb * 16 + gq, rowB = rowA + 8;
      if (!SCORE) {
        float mxA = -INFINITY, mxB = -INFINITY;
#pragma unroll
        for (int n = 0; n < 8; ++n) {
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int t = tbase + n * 8 + 2 * cq + e;
            const bool ok = t < p.Tm;
            acc[n][e] = ok ? acc[n][e] * p.scale_log2 : -INFINITY;
            acc[n][2 + e] = ok ? acc[n][2 + e] * p.scale_log2 : -INFINITY;
            mxA = fmaxf(mxA, acc[n][e]);
            mxB = fmaxf(mxB, acc[n][2 + e]);
          }
        }
        mxA = fmaxf(mxA, __shfl_xor_sync(0xffffffffu, mxA, 1));
        mxA = fmaxf(mxA, __shfl_xor_sync(0xffffffffu, mxA, 2));
        mxB = fmaxf(mxB, __shfl_xor_sync(0xffffffffu, mxB, 1));
        mxB = fmaxf(mxB, __shfl_xor_sync(0xffffffffu, mxB, 2));
        const float mA = fmaxf(m_s[rowA], mxA), mB = fmaxf(m_s[rowB], mxB);
        float sA = 0.f, sB = 0.f;
#pragma unroll
        for (int n = 0; n < 8; ++n) {
          sA += exp2f(acc[n][0] - mA) + exp2f(acc[n][1] - mA);
          sB += exp2f(acc[n][2] - mB) + exp2f(acc[n][3] - mB);
        }
        sA += __shfl_xor_sync(0xffffffffu, sA, 1);
        sA += __shfl_xor_sync(0xffffffffu, sA, 2);
        sB += __shfl_xor_sync(0xffffffffu, sB, 1);
        sB += __shfl_xor_sync(0xffffffffu, sB, 2);
        __syncwarp();
        if (cq == 0) {
          l_s[rowA] = l_s[rowA] * exp2f(m_s[rowA] - mA) + sA;
          l_s[rowB] = l_s[rowB] * exp2f(m_s[rowB] - mB) + sB;
          m_s[rowA] = mA;
          m_s[rowB] = mB;
        }
        __syncwarp();
      } else {
        const int hq_base = g * p.n_rep;
        // global row index = (hq)*Wp + i ; local row = r*Wp + i
        const int grA = hq_base * p.Wp + rowA, grB = hq_base * p.Wp + rowB;
        const float2 stA = p.ml[grA], stB = p.ml[grB];
        const bool validA = (rowA % p.Wp) < p.W, validB = (rowB % p.Wp) < p.W;
        const float invA = validA ? 1.f / stA.y : 0.f, invB = validB ? 1.f / stB.y : 0.f;
        float colsum[8][2];
#pragma unroll
        for (int n = 0; n < 8; ++n) {
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const float pa = validA ? exp2f(acc[n][e] * p.scale_log2 - stA.x) * invA : 0.f;
            const float pb = validB ? exp2f(acc[n][2 + e] * p.scale_log2 - stB.x) * invB : 0.f;
            float v = pa + pb;
            // sum over the 8 row pairs of the 16-row block (lanes with equal cq)
            v += __shfl_xor_sync(0xffffffffu, v, 4);
            v += __shfl_xor_sync(0xffffffffu, v, 8);
            v += __shfl_xor_sync(0xffffffffu, v, 16);
            colsum[n][e] = v;
          }
        }
        if (gq == 0) {
#pragma unroll
          for (int n = 0; n < 8; ++n) {
            cs[rb * kTileTok + n * 8 + 2 * cq] = colsum[n][0];
            cs[rb * kTileTok + n * 8 + 2 * cq + 1] = colsum[n][1];
          }
        }
      }
    }
    __syncthreads();
    if (SCORE) {
      // mean over the W window rows of each head (fixed rb order), max over heads
      const int rb_per_head = p.Wp / 16;
      const float invW = 1.f / static_cast<float>(p.W);
      for (int t = tid; t < kTileTok; t += blockDim.x) {
        const int tt = tbase + t;
        if (tt >= p.Tm) continue;
        float best = -INFINITY;
        for (int r = 0; r < p.n_rep; ++r) {
          float ssum = 0.f;
          for (int j = 0; j < rb_per_head; ++j) ssum += cs[(r * rb_per_head + j) * kTileTok + t];
          best = fmaxf(best, ssum * invW);
        }
        p.headmax[static_cast<int64_t>(g) * p.Tm + tt] = best;
      }
      __syncthreads();
    }
  }
  if (!SCORE) {
    __syncthreads();
    for (int r = tid; r < rows; r += blockDim.x) {
      const int grow = g * p.n_rep * p.Wp + r;
      p.ml_part[static_cast<int64_t>(grow) * p.n_chunks + chunk] = make_float2(m_s[r], l_s[r]);
    }
  }
}

// One warp per window row: (m, l) over the row's chunks, coalesced, fixed order
// (lane-strided partial then a fixed shuffle tree).
__global__ void stats_reduce_kernel(const float2* ml_part, float2* ml, int nrows, int n_chunks) {
  const int r = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (r >= nrows) return;
  const float2* src = ml_part + static_cast<int64_t>(r) * n_chunks;
  float m = -INFINITY;
  for (int c = lane; c < n_chunks; c += 32) m = fmaxf(m, src[c].x);
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  float l = 0.f;
  for (int c = lane; c < n_chunks; c += 32) l += src[c].y * exp2f(src[c].x - m);
  for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
  if (lane == 0) ml[r] = make_float2(m, l);
}

// Block scores: a CTA of 256 threads covers kBlkPerCta blocks plus one halo
// block on each side.  Thread = token: max over kv heads (coalesced rows of
// headmax), 16-token sums by a fixed shuffle tree, then optional max-pool 3.
// per_head: no max over kv heads; KV head blockIdx.y writes its own row
// out[blockIdx.y][N].
constexpr int kBlkPerCta = 14;  // (14 + 2) blocks x 16 tokens = 256 threads
__global__ void __launch_bounds__(256) block_reduce_kernel(const float* headmax, float* out, int Hkv, int slots,
                                                           int Tm, int N, int smooth, int per_head) {
  pdl_wait();
  __shared__ float raw[kBlkPerCta + 2];
  const int b0 = blockIdx.x * kBlkPerCta - 1;  // first (halo) block
  const int t = threadIdx.x;
  const int blk = b0 + t / kPage;
  const int tok = blk * kPage + (t % kPage);
  float v = 0.f;
  if (blk >= 0 && blk < N) {
    float mx = -INFINITY;
    // rows g*slots .. g*slots+slots-1 belong to KV group g
    const int r0 = per_head ? static_cast<int>(blockIdx.y) * slots : 0;
    const int r1 = per_head ? r0 + slots : Hkv * slots;
    for (int r = r0; r < r1; ++r) mx = fmaxf(mx, headmax[static_cast<int64_t>(r) * Tm + tok]);
    v = mx;
  }
  for (int o = 1; o < kPage; o <<= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if ((t % kPage) == 0) raw[t / kPage] = v;
  __syncthreads();
  if (t < kBlkPerCta) {
    const int n = b0 + 1 + t;
    if (n < N) {
      float r = raw[t + 1];
      const bool pool = smooth == 2 || (smooth == 1 && N >= 3);
      if (pool) {
        if (n > 0) r = fmaxf(r, raw[t]);
        if (n + 1 < N) r = fmaxf(r, raw[t + 2]);
      }
      out[static_cast<int64_t>(blockIdx.y) * N + n] = r;
    }
  }
}

// ---------------------------------------------------------------------------
// Top-k: one CTA bitonic-sorts 64-bit keys (descending score, ascending index)
// and emits the k smallest-keyed indices in ascending index order.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t desc_key(float f) {
  uint32_t u = __float_as_uint(f);
  if (f != f) u = 0x7fc00000u;  // canonical NaN ranks above +inf (torch.topk)
  const uint32_t ord = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return ~ord;
}

// Exclusive block scan of per-thread counts (threads own contiguous index ranges).
__device__ int block_exclusive_scan(int local, int* wsum) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = blockDim.x >> 5;
  int incl = local;
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  __syncthreads();
  if (lane == 31) wsum[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    const int w = lane < nw ? wsum[lane] : 0;
    int wi = w;
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, wi, o);
      if (lane >= o) wi += y;
    }
    wsum[lane] = wi - w;
  }
  __syncthreads();
  return wsum[warp] + incl - local;
}

// Top-k by radix select on 32-bit order keys (smaller key = higher score):
// four 8-bit passes find the exact k-th smallest key T and how many keys equal
// to T are still needed; the selection is every key < T plus the first of the
// keys == T in index order (ties -> lowest index), written in ascending index
// order by an ordered compaction.
__global__ void __launch_bounds__(1024) topk_select_kernel(const float* scores, int n, int k, int32_t* selected) {
  extern __shared__ __align__(128) uint8_t smem[];
  pdl_wait();
  scores += static_cast<int64_t>(blockIdx.x) * n;  // one row of a batch per CTA
  selected += static_cast<int64_t>(blockIdx.x) * k;
  uint32_t* key = reinterpret_cast<uint32_t*>(smem);
  __shared__ int hist[256];
  __shared__ int wsum[32];
  __shared__ uint32_t s_prefix;
  __shared__ int s_need;
  const int tid = threadIdx.x, nt = blockDim.x;
  for (int i = tid; i < n; i += nt) key[i] = desc_key(scores[i]);
  if (tid == 0) {
    s_prefix = 0;
    s_need = k;
  }
  uint32_t mask = 0;
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int b = tid; b < 256; b += nt) hist[b] = 0;
    __syncthreads();
    const uint32_t prefix = s_prefix;
    for (int i = tid; i < n; i += nt) {
      const uint32_t kv = key[i];
      if ((kv & mask) == prefix) atomicAdd(&hist[(kv >> shift) & 255u], 1);
    }
    __syncthreads();
    if (tid < 32) {  // warp 0: bin where the cumulative count reaches s_need
      const int need = s_need;
      int c[8], run = 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        c[j] = hist[tid * 8 + j];
        run += c[j];
      }
      int incl = run;
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, incl, o);
        if (tid >= o) incl += y;
      }
      int before = incl - run;
      const bool mine = before < need && incl >= need;
      if (mine) {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          if (before + c[j] >= need) {
            s_prefix = prefix | (static_cast<uint32_t>(tid * 8 + j) << shift);
            s_need = need - before;
            break;
          }
          before += c[j];
        }
      }
    }
    mask |= 255u << shift;
    __syncthreads();
  }
  const uint32_t T = s_prefix;
  const int need_eq = s_need;
  const int per = (n + nt - 1) / nt;
  const int beg = min(tid * per, n), end = min(beg + per, n);
  int eq_local = 0;
  for (int i = beg; i < end; ++i) eq_local += key[i] == T;
  int eq_rank = block_exclusive_scan(eq_local, wsum);
  int sel_local = 0;
  for (int i = beg; i < end; ++i) {
    const uint32_t kv = key[i];
    const bool take = kv < T || (kv == T && eq_rank++ < need_eq);
    sel_local += take;
  }
  int pos = block_exclusive_scan(sel_local, wsum);
  eq_rank = block_exclusive_scan(eq_local, wsum);
  for (int i = beg; i < end; ++i) {
    const uint32_t kv = key[i];
    const bool take = kv < T || (kv == T && eq_rank++ < need_eq);
    if (take) selected[pos++] = i;
  }
}

// ---------------------------------------------------------------------------
// Compacting writeback: destination token p of the compacted sequence.
// ---------------------------------------------------------------------------
__device__ __forceinline__ int64_t compact_src_token(int p, int L, int sink, int obs, int kb,
                                                     const int32_t* selected) {
  if (kb < 0) return p < L ? p : -1;  // uncompressed copy
  if (p < sink) return p;
  const int mid_end = sink + kPage * kb;
  if (p < mid_end) {
    const int r = (p - sink) / kPage, o = (p - sink) % kPage;
    const int64_t t = sink + static_cast<int64_t>(kPage) * selected[r] + o;
    return t < L - obs ? t : -1;  // -1: zero padding of a partial mid block
  }
  return static_cast<int64_t>(L - obs) + (p - mid_end);
}

template <typename V>
__global__ void page_compact_kernel(const uint8_t* k_src, const uint8_t* v_src, uint8_t* k_pool, uint8_t* v_pool,
                                    const int32_t* selected, int kb, const int32_t* dst_pages, int L, int sink,
                                    int obs, int eff_len, int Hkv, int row_bytes, int64_t src_sh_b,
                                    int64_t src_st_b, int64_t page_stride_b, int64_t dst_st_b, int64_t dst_sh_b,
                                    int64_t sel_stride_h) {
  pdl_wait();
  const int j = blockIdx.x;  // destination page
  const bool is_v = blockIdx.y == 1;
  const uint8_t* src = is_v ? v_src : k_src;
  uint8_t* dst = (is_v ? v_pool : k_pool) + static_cast<int64_t>(dst_pages[j]) * page_stride_b;
  const int vec_per_row = row_bytes / static_cast<int>(sizeof(V));
  const int total = kPage * Hkv * vec_per_row;
  constexpr int kMaxRows = 256;  // (slot, head) rows of one page staged in shared memory
  if (vec_per_row <= static_cast<int>(blockDim.x) && blockDim.x % vec_per_row == 0 && kPage * Hkv <= kMaxRows) {
    // The source and destination offsets of each row (slot, head) are computed once, by one
    // thread, into shared memory (the vec_per_row threads that copy a row's columns would
    // otherwise each redo the source-token arithmetic); then each thread keeps one column vi
    // of the rows it visits, and the loads of a batch of rows go out before its stores.
    __shared__ int64_t s_src[kMaxRows];  // byte offset in src, -1 = zero row, -2 = slot past eff_len
    __shared__ int64_t s_dst[kMaxRows];
    const int nrows = kPage * Hkv;
    for (int rh = threadIdx.x; rh < nrows; rh += blockDim.x) {
      const int h = rh % Hkv, slot = rh / Hkv;
      const int p = j * kPage + slot;
      int64_t so = -2;
      if (p < eff_len) {  // slots past the compacted length stay untouched
        const int64_t t = compact_src_token(p, L, sink, obs, kb, selected + h * sel_stride_h);
        so = t >= 0 ? h * src_sh_b + t * src_st_b : -1;
      }
      s_src[rh] = so;
      s_dst[rh] = slot * dst_st_b + h * dst_sh_b;
    }
    __syncthreads();
    constexpr int kBatch = 8;
    const int vi = threadIdx.x % vec_per_row;
    const int rstep = blockDim.x / vec_per_row;
    for (int r0 = threadIdx.x / vec_per_row; r0 < nrows; r0 += rstep * kBatch) {
      V val[kBatch];
      int64_t so[kBatch];
#pragma unroll
      for (int u = 0; u < kBatch; ++u) {
        const int rh = r0 + u * rstep;
        so[u] = rh < nrows ? s_src[rh] : -2;
        if (so[u] >= 0) {
          val[u] = __ldg(reinterpret_cast<const V*>(src + so[u]) + vi);
        } else {
          memset(&val[u], 0, sizeof(V));
        }
      }
#pragma unroll
      for (int u = 0; u < kBatch; ++u) {
        const int rh = r0 + u * rstep;
        if (so[u] != -2) *(reinterpret_cast<V*>(dst + s_dst[rh]) + vi) = val[u];
      }
    }
    return;
  }
  for (int i = threadIdx.x; i < total; i += blockDim.x) {
    const int vi = i % vec_per_row;
    const int rh = i / vec_per_row;
    const int h = rh % Hkv, slot = rh / Hkv;
    const int p = j * kPage + slot;
    if (p >= eff_len) continue;  // slots past the compacted length stay untouched
    const int64_t t = compact_src_token(p, L, sink, obs, kb, selected + h * sel_stride_h);
    V val;
    if (t >= 0) {
      val = *reinterpret_cast<const V*>(src + h * src_sh_b + t * src_st_b + vi * sizeof(V));
    } else {
      memset(&val, 0, sizeof(V));
    }
    *reinterpret_cast<V*>(dst + slot * dst_st_b + h * dst_sh_b + vi * sizeof(V)) = val;
  }
}

// ---------------------------------------------------------------------------
// Page gather / scatter between a pool and a packed buffer.
// ---------------------------------------------------------------------------
template <typename V, bool GATHER>
__global__ void page_move_kernel(const uint8_t* src, uint8_t* dst, const int32_t* ids, int64_t page_bytes,
                                 int64_t page_stride_b) {
  const int i = blockIdx.x;
  const int64_t pool_off = static_cast<int64_t>(ids[i]) * page_stride_b;
  const int64_t pack_off = static_cast<int64_t>(i) * page_bytes;
  const uint8_t* s = src + (GATHER ? pool_off : pack_off);
  uint8_t* d = dst + (GATHER ? pack_off : pool_off);
  const int64_t nvec = page_bytes / static_cast<int64_t>(sizeof(V));
  for (int64_t v = threadIdx.x; v < nvec; v += blockDim.x)
    reinterpret_cast<V*>(d)[v] = reinterpret_cast<const V*>(s)[v];
}

inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

struct ScoreWs {
  size_t ml_part, ml, headmax, total;
};
ScoreWs score_ws(int Hq, int W, int L, int sink, int obs) {
  const int Lm = L - sink - obs;
  const int N = (Lm + kPage - 1) / kPage;
  const int Tm = N * kPage;
  const int Wp = (W + 15) / 16 * 16;
  const int n_chunks = (Tm + kTileTok * kChunkTiles - 1) / (kTileTok * kChunkTiles);
  const int Hkv_max = Hq;  // upper bound for headmax rows (KV groups x head slots <= q heads)
  ScoreWs w;
  w.ml_part = 0;
  w.ml = align_up(sizeof(float2) * static_cast<size_t>(Hq) * Wp * n_chunks, 256);
  w.headmax = w.ml + align_up(sizeof(float2) * static_cast<size_t>(Hq) * Wp, 256);
  w.total = w.headmax + align_up(sizeof(float) * static_cast<size_t>(Hkv_max) * Tm, 256);
  return w;
}

template <typename T, int D>
int launch_score(ScoreParams& p, float* out, int N, int smooth, int per_head, cudaStream_t st) {
  const dim3 rgrid((N + kBlkPerCta - 1) / kBlkPerCta, per_head ? p.Hkv : 1);
  if constexpr (D == 128) {
    ScoreTcParams t{};
    t.k = p.k;
    t.q = p.q;
    t.Hkv = p.Hkv;
    t.n_rep = p.n_rep;
    t.W = p.W;
    t.Wp = p.Wp;
    t.Lm = p.Lm;
    t.Tm = p.Tm;
    t.sink = p.sink;
    t.k_sh = p.k_sh;
    t.k_st = p.k_st;
    t.q_sh = p.q_sh;
    t.q_st = p.q_st;
    t.scale_log2 = p.scale_log2;
    t.n_chunks = p.n_chunks;  // workspace capacity; pass 1 sets the ranges actually used
    t.ml_part = p.ml_part;
    t.ml = p.ml;
    t.headmax = p.headmax;
    const int dt = std::is_same<T, __nv_bfloat16>::value ? BPKV_BF16 : BPKV_F16;
    int rc = score_tc_pass(t, D, dt, 1, st);
    if (rc != BPKV_ERR_UNSUPPORTED) {
      if (rc != BPKV_OK) return rc;
      // (pass 2 merges the per-range row statistics itself: no stats_reduce launch)
      rc = score_tc_pass(t, D, dt, 2, st);
      if (rc != BPKV_OK) return rc;
      {
        const cudaError_t le = launch_pdl(block_reduce_kernel, rgrid, dim3(256), 0, st, (const float*)p.headmax, out,
                                          p.Hkv, t.hm_slots, p.Tm, N, smooth, per_head);
        if (le != cudaSuccess) {
          set_error("block_score_launch:%s", cudaGetErrorString(le));
          return BPKV_ERR_CUDA;
        }
      }
      BPKV_RETURN_LAUNCH("block_score_launch");
    }
  }
  const int rows = p.n_rep * p.Wp;
  const size_t smem = static_cast<size_t>(rows) * D * 2 + 2 * kTileTok * D * 2 +
                      sizeof(float) * max(rows / 16 * kTileTok, 2 * rows);
  if (smem > 227 * 1024) {
    set_error("block_score_shape_unsupported:window_rows_%d_head_dim_%d", rows, D);
    return BPKV_ERR_UNSUPPORTED;
  }
  auto k1 = score_tile_kernel<T, D, false>;
  auto k2 = score_tile_kernel<T, D, true>;
  cudaFuncSetAttribute(k1, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  cudaFuncSetAttribute(k2, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  dim3 grid(p.n_chunks, p.Hkv);
  k1<<<grid, kScoreWarps * 32, smem, st>>>(p);
  const int nrows = p.Hq * p.Wp;
  stats_reduce_kernel<<<(nrows * 32 + 255) / 256, 256, 0, st>>>(p.ml_part, p.ml, nrows, p.n_chunks);
  k2<<<grid, kScoreWarps * 32, smem, st>>>(p);
  block_reduce_kernel<<<rgrid, 256, 0, st>>>(p.headmax, out, p.Hkv, 1, p.Tm, N, smooth, per_head);
  BPKV_RETURN_LAUNCH("block_score_launch");
}

}  // namespace
}  // namespace bpkv

using namespace bpkv;

extern "C" BPKV_API size_t bpkv_block_score_workspace_size(int num_q_heads, int window, int L, int sink_len,
                                                           int obs_len) {
  if (num_q_heads <= 0 || window <= 0 || L - sink_len - obs_len <= 0) return 0;
  return score_ws(num_q_heads, window, L, sink_len, obs_len).total;
}

static int block_score_impl(const void* k, const void* q_obs, float* block_scores, int num_kv_heads,
                            int num_q_heads, int L, int window, int head_dim, int sink_len, int obs_len,
                            int64_t k_stride_h, int64_t k_stride_t, int64_t q_stride_h, int64_t q_stride_t,
                            float softmax_scale, int smooth, int dtype, void* workspace, size_t workspace_bytes,
                            void* stream, int per_head) {
  clear_error();
  BPKV_CHECK_ARG(num_kv_heads > 0 && num_q_heads > 0 && num_q_heads % num_kv_heads == 0,
                 "selected_writeback_bad_score_shape:gqa");
  BPKV_CHECK_ARG(window > 0 && head_dim > 0 && sink_len >= 0 && obs_len >= 0,
                 "selected_writeback_bad_score_shape:empty");
  BPKV_CHECK_ARG(L >= sink_len + obs_len + kPage, "selected_writeback_bad_score_shape:too_short_%d", L);
  BPKV_CHECK_ARG(k && q_obs && block_scores, "selected_writeback_bad_score_shape:null_pointer");
  if (dtype != BPKV_F16 && dtype != BPKV_BF16) {
    set_error("block_score_shape_unsupported:dtype_%d", dtype);
    return BPKV_ERR_UNSUPPORTED;
  }
  if (!(head_dim == 32 || head_dim == 64 || head_dim == 128 || head_dim == 256) || !aligned16(k) ||
      !aligned16(q_obs) || k_stride_h % 8 || k_stride_t % 8 || q_stride_h % 8 || q_stride_t % 8) {
    set_error("block_score_shape_unsupported:head_dim_%d_or_alignment", head_dim);
    return BPKV_ERR_UNSUPPORTED;
  }
  const ScoreWs w = score_ws(num_q_heads, window, L, sink_len, obs_len);
  if (workspace == nullptr || workspace_bytes < w.total) {
    set_error("block_score_workspace:need_%zu_bytes", w.total);
    return BPKV_ERR_WORKSPACE;
  }
  ScoreParams p;
  p.k = k;
  p.q = q_obs;
  p.Hkv = num_kv_heads;
  p.Hq = num_q_heads;
  p.n_rep = num_q_heads / num_kv_heads;
  p.L = L;
  p.W = window;
  p.Wp = (window + 15) / 16 * 16;
  p.D = head_dim;
  p.sink = sink_len;
  p.obs = obs_len;
  p.Lm = L - sink_len - obs_len;
  const int N = (p.Lm + kPage - 1) / kPage;
  p.Tm = N * kPage;
  p.n_chunks = (p.Tm + kTileTok * kChunkTiles - 1) / (kTileTok * kChunkTiles);
  p.k_sh = k_stride_h;
  p.k_st = k_stride_t;
  p.q_sh = q_stride_h;
  p.q_st = q_stride_t;
  p.scale_log2 = softmax_scale * 1.4426950408889634f;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  p.ml_part = reinterpret_cast<float2*>(ws + w.ml_part);
  p.ml = reinterpret_cast<float2*>(ws + w.ml);
  p.headmax = reinterpret_cast<float*>(ws + w.headmax);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
#define BPKV_SCORE(TY)                                                      \
  switch (head_dim) {                                                       \
    case 32: return launch_score<TY, 32>(p, block_scores, N, smooth, per_head, st);   \
    case 64: return launch_score<TY, 64>(p, block_scores, N, smooth, per_head, st);   \
    case 128: return launch_score<TY, 128>(p, block_scores, N, smooth, per_head, st); \
    default: return launch_score<TY, 256>(p, block_scores, N, smooth, per_head, st);  \
  }
  if (dtype == BPKV_BF16) {
    BPKV_SCORE(__nv_bfloat16)
  } else {
    BPKV_SCORE(__half)
  }
#undef BPKV_SCORE
}

extern "C" BPKV_API int bpkv_block_score(const void* k, const void* q_obs, float* block_scores, int num_kv_heads,
                                         int num_q_heads, int L, int window, int head_dim, int sink_len,
                                         int obs_len, int64_t k_stride_h, int64_t k_stride_t,
                                         int64_t q_stride_h, int64_t q_stride_t, float softmax_scale, int smooth,
                                         int dtype, void* workspace, size_t workspace_bytes, void* stream) {
  return block_score_impl(k, q_obs, block_scores, num_kv_heads, num_q_heads, L, window, head_dim, sink_len, obs_len,
                          k_stride_h, k_stride_t, q_stride_h, q_stride_t, softmax_scale, smooth, dtype, workspace,
                          workspace_bytes, stream, 0);
}

extern "C" BPKV_API int bpkv_block_score_per_kv_head(const void* k, const void* q_obs, float* block_scores,
                                                     int num_kv_heads, int num_q_heads, int L, int window,
                                                     int head_dim, int sink_len, int obs_len, int64_t k_stride_h,
                                                     int64_t k_stride_t, int64_t q_stride_h, int64_t q_stride_t,
                                                     float softmax_scale, int smooth, int dtype, void* workspace,
                                                     size_t workspace_bytes, void* stream) {
  return block_score_impl(k, q_obs, block_scores, num_kv_heads, num_q_heads, L, window, head_dim, sink_len, obs_len,
                          k_stride_h, k_stride_t, q_stride_h, q_stride_t, softmax_scale, smooth, dtype, workspace,
                          workspace_bytes, stream, 1);
}

extern "C" BPKV_API int bpkv_topk_select_batched(const float* scores, int n, int k, int batch, int32_t* selected,
                                                 void* stream) {
  clear_error();
  BPKV_CHECK_ARG(batch >= 0, "selected_writeback_topk_shape:batch_%d", batch);
  BPKV_CHECK_ARG(n >= 0 && k >= 0 && k <= n, "selected_writeback_topk_shape:n_%d_k_%d", n, k);
  BPKV_CHECK_ARG(n <= 49152, "selected_writeback_topk_shape:n_%d_exceeds_49152", n);
  if (k == 0) return BPKV_OK;
  BPKV_CHECK_ARG(scores && selected, "selected_writeback_topk_shape:null_pointer");
  const size_t smem = sizeof(uint32_t) * n;
  static bool raised[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (smem > 48 * 1024 && dev < 64 && !raised[dev]) {
    cudaFuncSetAttribute(topk_select_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         static_cast<int>(sizeof(uint32_t) * 49152));
    raised[dev] = true;
  }
  if (batch == 0) return BPKV_OK;
  const cudaError_t le = launch_pdl(topk_select_kernel, dim3(batch), dim3(1024), smem,
                                    static_cast<cudaStream_t>(stream), scores, n, k, selected);
  if (le != cudaSuccess) {
    set_error("topk_select_launch:%s", cudaGetErrorString(le));
    return BPKV_ERR_CUDA;
  }
  BPKV_RETURN_LAUNCH("topk_select_launch");
}

extern "C" BPKV_API int bpkv_topk_select(const float* scores, int n, int k, int32_t* selected, void* stream) {
  return bpkv_topk_select_batched(scores, n, k, 1, selected, stream);
}

static int page_compact_impl(const void* k_src, const void* v_src, void* k_pool, void* v_pool,
                             const int32_t* selected, int64_t sel_stride_h, int k_blocks, const int32_t* dst_pages,
                             int L, int sink_len, int obs_len, int num_kv_heads, int head_dim, int64_t src_stride_h,
                             int64_t src_stride_t, int64_t page_stride, int64_t dst_stride_t, int64_t dst_stride_h,
                             int dtype, void* stream) {
  clear_error();
  BPKV_CHECK_ARG(L > 0 && num_kv_heads > 0 && head_dim > 0 && sink_len >= 0 && obs_len >= 0,
                 "selected_writeback_shape:empty");
  BPKV_CHECK_ARG(k_blocks < 0 || L >= sink_len + obs_len, "selected_writeback_shape:too_short");
  BPKV_CHECK_ARG(k_src && v_src && k_pool && v_pool && dst_pages, "selected_writeback_shape:null_pointer");
  BPKV_CHECK_ARG(k_blocks <= 0 || selected != nullptr, "selected_writeback_shape:null_selected");
  const int esz = dtype == BPKV_F32 ? 4 : 2;
  BPKV_CHECK_ARG(dtype == BPKV_F32 || dtype == BPKV_F16 || dtype == BPKV_BF16, "selected_writeback_shape:dtype");
  const int eff_len = k_blocks < 0 ? L : sink_len + kPage * k_blocks + obs_len;
  const int n_pages = (eff_len + kPage - 1) / kPage;
  if (n_pages == 0) return BPKV_OK;
  const int row_bytes = head_dim * esz;
  const int64_t sh = src_stride_h * esz, stt = src_stride_t * esz, ps = page_stride * esz;
  const int64_t dt = dst_stride_t * esz, dh = dst_stride_h * esz;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  dim3 grid(n_pages, 2);
  const bool v16 = row_bytes % 16 == 0 && sh % 16 == 0 && stt % 16 == 0 && ps % 16 == 0 && dt % 16 == 0 &&
                   dh % 16 == 0 && aligned16(k_src) &&
                   aligned16(v_src) && aligned16(k_pool) && aligned16(v_pool);
  const uint8_t *ks = static_cast<const uint8_t*>(k_src), *vs = static_cast<const uint8_t*>(v_src);
  uint8_t *kp = static_cast<uint8_t*>(k_pool), *vp = static_cast<uint8_t*>(v_pool);
  if (v16)
    launch_pdl(page_compact_kernel<uint4>, grid, dim3(256), 0, st, ks, vs, kp, vp, selected, k_blocks, dst_pages, L, sink_len,
                                                     obs_len, eff_len, num_kv_heads, row_bytes, sh, stt, ps, dt, dh,
        sel_stride_h);
  else if (esz == 4)
    launch_pdl(page_compact_kernel<uint32_t>, grid, dim3(256), 0, st, ks, vs, kp, vp, selected, k_blocks, dst_pages, L, sink_len,
                                                        obs_len, eff_len, num_kv_heads, row_bytes, sh, stt, ps, dt, dh,
        sel_stride_h);
  else
    launch_pdl(page_compact_kernel<uint16_t>, grid, dim3(256), 0, st, ks, vs, kp, vp, selected, k_blocks, dst_pages, L, sink_len,
                                                        obs_len, eff_len, num_kv_heads, row_bytes, sh, stt, ps, dt, dh,
        sel_stride_h);
  BPKV_RETURN_LAUNCH("page_compact_launch");
}

extern "C" BPKV_API int bpkv_page_compact(const void* k_src, const void* v_src, void* k_pool, void* v_pool,
                                          const int32_t* selected, int k_blocks, const int32_t* dst_pages, int L,
                                          int sink_len, int obs_len, int num_kv_heads, int head_dim,
                                          int64_t src_stride_h, int64_t src_stride_t, int64_t page_stride,
                                          int64_t dst_stride_t, int64_t dst_stride_h, int dtype, void* stream) {
  return page_compact_impl(k_src, v_src, k_pool, v_pool, selected, 0, k_blocks, dst_pages, L, sink_len, obs_len,
                           num_kv_heads, head_dim, src_stride_h, src_stride_t, page_stride, dst_stride_t,
                           dst_stride_h, dtype, stream);
}

extern "C" BPKV_API int bpkv_page_compact_per_kv_head(const void* k_src, const void* v_src, void* k_pool,
                                                      void* v_pool, const int32_t* selected,
                                                      int64_t selected_stride_h, int k_blocks,
                                                      const int32_t* dst_pages, int L, int sink_len, int obs_len,
                                                      int num_kv_heads, int head_dim, int64_t src_stride_h,
                                                      int64_t src_stride_t, int64_t page_stride,
                                                      int64_t dst_stride_t, int64_t dst_stride_h, int dtype,
                                                      void* stream) {
  if (k_blocks > 0 && selected_stride_h < k_blocks) {
    clear_error();
    set_error("selected_writeback_shape:selected_stride_%lld", static_cast<long long>(selected_stride_h));
    return BPKV_ERR_SHAPE;
  }
  return page_compact_impl(k_src, v_src, k_pool, v_pool, selected, selected_stride_h, k_blocks, dst_pages, L,
                           sink_len, obs_len, num_kv_heads, head_dim, src_stride_h, src_stride_t, page_stride,
                           dst_stride_t, dst_stride_h, dtype, stream);
}

static int page_move(const void* src, void* dst, const int32_t* ids, int n_pages, int64_t page_elems,
                     int64_t page_stride, int dtype, void* stream, bool gather) {
  clear_error();
  BPKV_CHECK_ARG(n_pages >= 0 && page_elems > 0, "page_move_shape:empty");
  if (n_pages == 0) return BPKV_OK;
  BPKV_CHECK_ARG(src && dst && ids, "page_move_shape:null_pointer");
  const int esz = dtype == BPKV_F32 ? 4 : 2;
  const int64_t pb = page_elems * esz, ps = page_stride * esz;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const uint8_t* s = static_cast<const uint8_t*>(src);
  uint8_t* d = static_cast<uint8_t*>(dst);
  const bool v16 = pb % 16 == 0 && ps % 16 == 0 && aligned16(src) && aligned16(dst);
  if (gather) {
    if (v16) page_move_kernel<uint4, true><<<n_pages, 256, 0, st>>>(s, d, ids, pb, ps);
    else page_move_kernel<uint16_t, true><<<n_pages, 256, 0, st>>>(s, d, ids, pb, ps);
  } else {
    if (v16) page_move_kernel<uint4, false><<<n_pages, 256, 0, st>>>(s, d, ids, pb, ps);
    else page_move_kernel<uint16_t, false><<<n_pages, 256, 0, st>>>(s, d, ids, pb, ps);
  }
  BPKV_RETURN_LAUNCH("page_move_launch");
}

extern "C" BPKV_API int bpkv_page_gather(const void* pool, const int32_t* page_ids, int n_pages, void* packed,
                                         int64_t page_elems, int64_t page_stride, int dtype, void* stream) {
  return page_move(pool, packed, page_ids, n_pages, page_elems, page_stride, dtype, stream, true);
}

extern "C" BPKV_API int bpkv_page_scatter(const void* packed, const int32_t* page_ids, int n_pages, void* pool,
                                          int64_t page_elems, int64_t page_stride, int dtype, void* stream) {
  return page_move(packed, pool, page_ids, n_pages, page_elems, page_stride, dtype, stream, false);
}
