// Page16 split-KV GQA decode attention over the 16-token paged pool (sm_100a).
//
// Replaces the reference Triton kernel _page16_decode_kernel
// (core/page16_native.py:17-80), which runs one program per (request, q-head),
// walks every page serially and re-reads K/V once per q-head of a GQA group.
//
// Design (B200):
//  * Work split.  All requests' pages form one flattened list of
//    T = sum_b ceil(len_b/16) pages.  CTA c of G persistent CTAs owns pages
//    [floor(cT/G), floor((c+1)T/G)) - every SM gets the same number of pages
//    whatever the length mix.  A request cut by a range boundary yields one
//    partial (o, lse) per owning CTA in workspace slot (c + b) (unique, because
//    ranges are ordered), merged by a log-sum-exp combine kernel.
//  * One warp per KV head.  Each warp streams its head's 16-row K and V tiles
//    (16 x head_dim each) of every page through an NS-stage cp.async ring with
//    16-byte zero-filling copies (rows past len are zero, so stale pool data
//    never reaches the math), XOR-swizzled so ldmatrix is conflict free.
//    Warps never wait on each other: no block barrier in the main loop.
//  * All n_rep query heads of the group share one K/V read: S = Q_g K^T and
//    O += P V run on mma.m16n8k16 (fp32 accumulate) with the n_rep heads as
//    the M rows; P is reused straight from the S accumulators as the A
//    fragment.  Online softmax in the exp2 domain, row max / sum by quad
//    shuffles.  bf16 / fp16 P is split into a high and a low part (two MMAs),
//    keeping about 16 mantissa bits of each weight.
//  * Launches.  The combine is a programmatic dependent launch of the decode
//    grid: it is scheduled during the decode grid's tail (the decode CTAs
//    signal griddepcontrol.launch_dependents once their work is done) and
//    waits for the grid's completion before reading the partials.  It signals
//    its own dependents at its start.  A sequence split across GPUs replaces
//    the combine with split_kv_p2p_kernel (combine + NVLink exchange + merge in
//    one launch, also a programmatic dependent of the decode grid).
//  * Fused append (optional).  With k_new / v_new the warp that owns a
//    request's last page stores this step's token into the pool and takes its
//    row from k_new / v_new for the math, so append + decode is one launch.
#include <mutex>
#include <type_traits>

#include <string.h>

#include "common.cuh"
#include "peer_words.cuh"

namespace bpkv {
namespace {

struct DecodeParams {
  const void* q;
  const void* k;
  const void* v;
  const int32_t* bt;
  const int32_t* lens;
  void* out;
  float* lse_out;
  int32_t* g_prefix;  // workspace: prefix[B+1] written by CTA (0,0)
  float* part_lse;    // workspace: [slots][Hq]
  float* part_o;      // workspace: [slots][Hq][D]
  int B, Hq, Hkv, D, max_blocks, n_rep;
  int64_t q_sb, q_sh, page_stride, bt_sb;
  float scale;        // softmax scale
  float scale_log2;   // softmax scale * log2(e)
  // fused decode-token append (null = off): row [batch][h_kv][d] written at token len-1
  const void* k_new;
  const void* v_new;
  int64_t new_sb;
  // split-KV across GPUs: every CTA writes its fp32 partial to its slot (no direct
  // T output even for a request a single CTA owns), for the fused exchange kernel
  int partials_only;
  int num_splits;  // CTAs over the flattened page list; 0 = one per SM (per KV-head group)
};

constexpr float kLn2 = 0.6931471805599453f;

__device__ __forceinline__ int npages_of(const DecodeParams& p, int b) {
  int len = __ldg(p.lens + b);
  if (len <= 0) return 0;
  int np = (len + kPage - 1) / kPage;
  return np < p.max_blocks ? np : p.max_blocks;
}

__device__ __forceinline__ int eff_len(const DecodeParams& p, int b) {
  int len = __ldg(p.lens + b);
  int cap = p.max_blocks * kPage;
  return len < cap ? len : cap;
}

// Block-wide exclusive scan of per-request page counts into prefix[0..B].
__device__ void build_prefix(const DecodeParams& p, int* prefix) {
  __shared__ int wsum[32];
  const int nt = blockDim.x, tid = threadIdx.x;
  const int lane = tid & 31, warp = tid >> 5, nw = (nt + 31) >> 5;
  const int per = (p.B + nt - 1) / nt;
  const int beg = tid * per;
  const int end = min(beg + per, p.B);
  int local = 0;
  for (int i = beg; i < end; ++i) local += npages_of(p, i);
  int incl = local;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    int y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  if (lane == 31) wsum[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    int w = lane < nw ? wsum[lane] : 0;
    int wi = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int y = __shfl_up_sync(0xffffffffu, wi, o);
      if (lane >= o) wi += y;
    }
    wsum[lane] = wi - w;
    if (lane == 31) prefix[p.B] = wi;
  }
  __syncthreads();
  int run = wsum[warp] + incl - local;
  for (int i = beg; i < end; ++i) {
    prefix[i] = run;
    run += npages_of(p, i);
  }
  __syncthreads();
}

// Largest b with prefix[b] <= s  (s < prefix[B]).
__device__ __forceinline__ int find_request(const int* prefix, int B, int64_t s) {
  int lo = 0, hi = B;  // invariant prefix[lo] <= s < prefix[hi]
  while (hi - lo > 1) {
    int mid = (lo + hi) >> 1;
    if (prefix[mid] <= s) lo = mid; else hi = mid;
  }
  return lo;
}

// ---------------------------------------------------------------------------
// Tensor-core kernel: bf16 / fp16, head_dim in {64,128,256}, n_rep <= 16.
// ---------------------------------------------------------------------------
template <typename T, int D, int NW, int NS>
__global__ void __launch_bounds__(NW * 32, 1) page16_decode_mma_kernel(DecodeParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  constexpr int ROWB = D * 2;       // bytes of one token row of one head
  constexpr int TILEB = 16 * ROWB;  // one page, one head, K (or V)
  constexpr int STAGEB = 2 * TILEB;
  constexpr int CH = D / 8;                  // 16-byte chunks per row
  constexpr int PER_LANE = 16 * CH / 32;     // chunks per lane per tile
  constexpr int KS = D / 16;                 // mma k-steps over head_dim
  constexpr int NT = D / 8;                  // 8-wide output column tiles

  int* prefix = reinterpret_cast<int*>(smem + NW * NS * STAGEB);
  build_prefix(p, prefix);
  const int B = p.B;
  const int64_t total = prefix[B];
  const int G = gridDim.x, c = blockIdx.x;
  if (c == 0 && blockIdx.y == 0) {
    for (int i = threadIdx.x; i <= B; i += blockDim.x) p.g_prefix[i] = prefix[i];
  }
  if (total == 0) return;
  const int64_t s = range_start(c, total, G), e = range_start(c + 1, total, G);
  if (s >= e) return;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.y * NW + warp;  // kv head of this warp
  if (h >= p.Hkv) return;

  const T* __restrict__ kg = reinterpret_cast<const T*>(p.k);
  const T* __restrict__ vg = reinterpret_cast<const T*>(p.v);
  const uint32_t ring = smem_u32(smem + warp * NS * STAGEB);
  const int g = lane >> 2, cq = lane & 3;

  // ---- loader ------------------------------------------------------------
  auto issue = [&](int64_t fp, int b, int stage) {
    const int j = static_cast<int>(fp - prefix[b]);
    const int page = __ldg(p.bt + static_cast<int64_t>(b) * p.bt_sb + j);
    const int len_b = eff_len(p, b);
    const int valid_rows = len_b - j * kPage;  // >= 1
    // fused append: this step's token (position len-1) lives in the request's last page; its row
    // comes from k_new / v_new and is also stored to the pool page (no other CTA reads that page)
    const bool last_page = j == prefix[b + 1] - prefix[b] - 1;
    const int tok_new = (p.k_new != nullptr && last_page && __ldg(p.lens + b) == len_b) ? valid_rows - 1 : -1;
    const int64_t base = static_cast<int64_t>(page) * p.page_stride + static_cast<int64_t>(h) * D;
    const uint32_t sk = ring + stage * STAGEB;
    const uint32_t sv = sk + TILEB;
#pragma unroll
    for (int r = 0; r < PER_LANE; ++r) {
      const int ci = lane + 32 * r;
      const int tok = ci / CH, ch = ci % CH;
      const bool ok = tok < valid_rows;
      const int64_t off = base + static_cast<int64_t>(tok) * p.Hkv * D + ch * 8;
      const uint32_t so = tok * ROWB + ((ch ^ (tok & 7)) << 4);
      if (tok == tok_new) {
        const int64_t noff = static_cast<int64_t>(b) * p.new_sb + static_cast<int64_t>(h) * D + ch * 8;
        const T* kn = reinterpret_cast<const T*>(p.k_new) + noff;
        const T* vn = reinterpret_cast<const T*>(p.v_new) + noff;
        cp_async16(sk + so, kn, true);
        cp_async16(sv + so, vn, true);
        *reinterpret_cast<uint4*>(static_cast<T*>(const_cast<void*>(p.k)) + off) = *reinterpret_cast<const uint4*>(kn);
        *reinterpret_cast<uint4*>(static_cast<T*>(const_cast<void*>(p.v)) + off) = *reinterpret_cast<const uint4*>(vn);
        continue;
      }
      cp_async16(sk + so, ok ? (const void*)(kg + off) : (const void*)kg, ok);
      cp_async16(sv + so, ok ? (const void*)(vg + off) : (const void*)vg, ok);
    }
  };

  int b0 = find_request(prefix, B, s);
  int64_t ld_p = s;
  int ld_b = b0;
#pragma unroll
  for (int i = 0; i < NS - 1; ++i) {
    if (ld_p < e) {
      while (prefix[ld_b + 1] <= ld_p) ++ld_b;
      issue(ld_p, ld_b, i);
      ++ld_p;
    }
    cp_async_commit();
  }

  // ---- per-request state -------------------------------------------------
  uint32_t qa[KS][4];
  float acc[NT][4];
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  int cur_b = -1, cur_len = 0;
  int64_t seg_first = 0;
  const int row0 = g, row1 = g + 8;
  const bool r0ok = row0 < p.n_rep, r1ok = row1 < p.n_rep;

  auto load_q = [&](int b) {
    const T* qb = reinterpret_cast<const T*>(p.q) + static_cast<int64_t>(b) * p.q_sb;
    const T* q0 = qb + static_cast<int64_t>(h * p.n_rep + row0) * p.q_sh;
    const T* q1 = qb + static_cast<int64_t>(h * p.n_rep + row1) * p.q_sh;
#pragma unroll
    for (int ks = 0; ks < KS; ++ks) {
      const int col = ks * 16 + 2 * cq;
      qa[ks][0] = r0ok ? *reinterpret_cast<const uint32_t*>(q0 + col) : 0u;
      qa[ks][1] = r1ok ? *reinterpret_cast<const uint32_t*>(q1 + col) : 0u;
      qa[ks][2] = r0ok ? *reinterpret_cast<const uint32_t*>(q0 + col + 8) : 0u;
      qa[ks][3] = r1ok ? *reinterpret_cast<const uint32_t*>(q1 + col + 8) : 0u;
    }
  };

  auto finish = [&](int b, int64_t seg_end) {
    float L0 = l0 + __shfl_xor_sync(0xffffffffu, l0, 1);
    L0 += __shfl_xor_sync(0xffffffffu, L0, 2);
    float L1 = l1 + __shfl_xor_sync(0xffffffffu, l1, 1);
    L1 += __shfl_xor_sync(0xffffffffu, L1, 2);
    const float inv0 = 1.f / L0, inv1 = 1.f / L1;
    const float lse0 = (m0 + __log2f(L0)) * kLn2;
    const float lse1 = (m1 + __log2f(L1)) * kLn2;
    const bool whole = !p.partials_only && seg_first == prefix[b] && seg_end == prefix[b + 1];
    const int hq0 = h * p.n_rep + row0, hq1 = h * p.n_rep + row1;
    if (whole) {
      T* ob = reinterpret_cast<T*>(p.out) + static_cast<int64_t>(b) * p.Hq * D;
#pragma unroll
      for (int n = 0; n < NT; ++n) {
        const int col = n * 8 + 2 * cq;
        if (r0ok)
          *reinterpret_cast<uint32_t*>(ob + static_cast<int64_t>(hq0) * D + col) =
              pack2<T>(acc[n][0] * inv0, acc[n][1] * inv0);
        if (r1ok)
          *reinterpret_cast<uint32_t*>(ob + static_cast<int64_t>(hq1) * D + col) =
              pack2<T>(acc[n][2] * inv1, acc[n][3] * inv1);
      }
      if (p.lse_out != nullptr && cq == 0) {
        if (r0ok) p.lse_out[static_cast<int64_t>(b) * p.Hq + hq0] = lse0;
        if (r1ok) p.lse_out[static_cast<int64_t>(b) * p.Hq + hq1] = lse1;
      }
    } else {
      const int64_t slot = static_cast<int64_t>(blockIdx.x) + b;
      float* po = p.part_o + slot * p.Hq * D;
#pragma unroll
      for (int n = 0; n < NT; ++n) {
        const int col = n * 8 + 2 * cq;
        if (r0ok)
          *reinterpret_cast<float2*>(po + static_cast<int64_t>(hq0) * D + col) =
              make_float2(acc[n][0] * inv0, acc[n][1] * inv0);
        if (r1ok)
          *reinterpret_cast<float2*>(po + static_cast<int64_t>(hq1) * D + col) =
              make_float2(acc[n][2] * inv1, acc[n][3] * inv1);
      }
      if (cq == 0) {
        if (r0ok) p.part_lse[slot * p.Hq + hq0] = lse0;
        if (r1ok) p.part_lse[slot * p.Hq + hq1] = lse1;
      }
    }
  };

  int cb = b0;
  for (int64_t fp = s; fp < e; ++fp) {
    const int it = static_cast<int>(fp - s);
    if (ld_p < e) {
      while (prefix[ld_b + 1] <= ld_p) ++ld_b;
      issue(ld_p, ld_b, (it + NS - 1) % NS);
      ++ld_p;
    }
    cp_async_commit();

    while (prefix[cb + 1] <= fp) ++cb;
    if (cb != cur_b) {
      if (cur_b >= 0) finish(cur_b, fp);
      cur_b = cb;
      cur_len = eff_len(p, cb);
      seg_first = fp;
      load_q(cb);
#pragma unroll
      for (int n = 0; n < NT; ++n) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.f;
      m0 = m1 = -INFINITY;
      l0 = l1 = 0.f;
    }

    cp_async_wait<NS - 1>();
    __syncwarp();

    const uint32_t sk = ring + (it % NS) * STAGEB;
    const uint32_t sv = sk + TILEB;
    // ---- S = Q K^T  (rows: q heads, cols: 16 tokens as two n-tiles) ----
    float s0[4] = {0.f, 0.f, 0.f, 0.f}, s1[4] = {0.f, 0.f, 0.f, 0.f};
    {
      const int mi = lane >> 3, rr = lane & 7;
      const int tok = rr + 8 * (mi >> 1);
#pragma unroll
      for (int ks = 0; ks < KS; ++ks) {
        const int ch = 2 * ks + (mi & 1);
        uint32_t b0r, b1r, b2r, b3r;
        ldmatrix_x4(sk + tok * ROWB + ((ch ^ rr) << 4), b0r, b1r, b2r, b3r);
        mma16816<T>(s0, qa[ks], b0r, b1r);
        mma16816<T>(s1, qa[ks], b2r, b3r);
      }
    }
    // ---- online softmax (log2 domain) ----
    const int tbase = static_cast<int>(fp - prefix[cb]) * kPage;
    const int t0 = tbase + 2 * cq, t1 = t0 + 8;
    float x[8];
    x[0] = (t0 < cur_len) ? s0[0] * p.scale_log2 : -INFINITY;
    x[1] = (t0 + 1 < cur_len) ? s0[1] * p.scale_log2 : -INFINITY;
    x[2] = (t0 < cur_len) ? s0[2] * p.scale_log2 : -INFINITY;
    x[3] = (t0 + 1 < cur_len) ? s0[3] * p.scale_log2 : -INFINITY;
    x[4] = (t1 < cur_len) ? s1[0] * p.scale_log2 : -INFINITY;
    x[5] = (t1 + 1 < cur_len) ? s1[1] * p.scale_log2 : -INFINITY;
    x[6] = (t1 < cur_len) ? s1[2] * p.scale_log2 : -INFINITY;
    x[7] = (t1 + 1 < cur_len) ? s1[3] * p.scale_log2 : -INFINITY;
    float mx0 = fmaxf(fmaxf(x[0], x[1]), fmaxf(x[4], x[5]));
    float mx1 = fmaxf(fmaxf(x[2], x[3]), fmaxf(x[6], x[7]));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
    const float a0 = fast_exp2(m0 - mn0), a1 = fast_exp2(m1 - mn1);
    m0 = mn0;
    m1 = mn1;
    float pr[8];
    pr[0] = fast_exp2(x[0] - mn0);
    pr[1] = fast_exp2(x[1] - mn0);
    pr[2] = fast_exp2(x[2] - mn1);
    pr[3] = fast_exp2(x[3] - mn1);
    pr[4] = fast_exp2(x[4] - mn0);
    pr[5] = fast_exp2(x[5] - mn0);
    pr[6] = fast_exp2(x[6] - mn1);
    pr[7] = fast_exp2(x[7] - mn1);
    l0 = l0 * a0 + (pr[0] + pr[1] + pr[4] + pr[5]);
    l1 = l1 * a1 + (pr[2] + pr[3] + pr[6] + pr[7]);
#pragma unroll
    for (int n = 0; n < NT; ++n) {
      acc[n][0] *= a0;
      acc[n][1] *= a0;
      acc[n][2] *= a1;
      acc[n][3] *= a1;
    }
    uint32_t pa[4], pl[4];
    split2<T>(pr[0], pr[1], pa[0], pl[0]);
    split2<T>(pr[2], pr[3], pa[1], pl[1]);
    split2<T>(pr[4], pr[5], pa[2], pl[2]);
    split2<T>(pr[6], pr[7], pa[3], pl[3]);
    // ---- O += P V ----
    {
      const int mi = lane >> 3, rr = lane & 7;
      const int tok = rr + 8 * (mi & 1);
#pragma unroll
      for (int dt = 0; dt < D / 16; ++dt) {
        const int ch = 2 * dt + (mi >> 1);
        uint32_t b0r, b1r, b2r, b3r;
        ldmatrix_x4_trans(sv + tok * ROWB + ((ch ^ rr) << 4), b0r, b1r, b2r, b3r);
        mma16816<T>(acc[2 * dt], pa, b0r, b1r);
        mma16816<T>(acc[2 * dt + 1], pa, b2r, b3r);
        if constexpr (SplitP<T>::value) {
          mma16816<T>(acc[2 * dt], pl, b0r, b1r);
          mma16816<T>(acc[2 * dt + 1], pl, b2r, b3r);
        }
      }
    }
    __syncwarp();
  }
  cp_async_wait<0>();
  if (cur_b >= 0) finish(cur_b, e);
  // the combine kernel (launched with programmatic stream serialization) may start its
  // launch now; it still waits for this whole grid to finish before reading the partials
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---------------------------------------------------------------------------
// Generic CUDA-core kernel: any dtype (fp32 included), head_dim <= 256, any
// GQA ratio.  Same work split and partial slots as the tensor-core kernel.
// One warp per query head at a time; fp32 math with accurate expf.
// ---------------------------------------------------------------------------
template <typename T, int NW>
__global__ void __launch_bounds__(NW * 32) page16_decode_generic_kernel(DecodeParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  int* prefix = reinterpret_cast<int*>(smem);
  build_prefix(p, prefix);
  const int B = p.B;
  const int64_t total = prefix[B];
  const int G = gridDim.x, c = blockIdx.x;
  if (c == 0) {
    for (int i = threadIdx.x; i <= B; i += blockDim.x) p.g_prefix[i] = prefix[i];
  }
  if (total == 0) return;
  const int64_t s = range_start(c, total, G), e = range_start(c + 1, total, G);
  if (s >= e) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int D = p.D;
  const int nd = (D + 31) / 32;
  const T* kg = reinterpret_cast<const T*>(p.k);
  const T* vg = reinterpret_cast<const T*>(p.v);
  const int b0 = find_request(prefix, B, s);

  for (int hq = warp; hq < p.Hq; hq += NW) {
    const int h = hq / p.n_rep;
    float qv[8], acc[8];
    float m = -INFINITY, l = 0.f;
    int cur_b = -1, cur_len = 0;
    int64_t seg_first = 0;
    auto finish = [&](int b, int64_t seg_end) {
      const bool whole = !p.partials_only && seg_first == prefix[b] && seg_end == prefix[b + 1];
      const float inv = 1.f / l;
      const float lse = m + logf(l);
      if (whole) {
        T* ob = reinterpret_cast<T*>(p.out) + (static_cast<int64_t>(b) * p.Hq + hq) * D;
        for (int i = 0; i < nd; ++i) {
          const int d = lane + 32 * i;
          if (d < D) ob[d] = Elem<T>::from_f(acc[i] * inv);
        }
        if (p.lse_out != nullptr && lane == 0) p.lse_out[static_cast<int64_t>(b) * p.Hq + hq] = lse;
      } else {
        const int64_t slot = static_cast<int64_t>(blockIdx.x) + b;
        float* po = p.part_o + (slot * p.Hq + hq) * D;
        for (int i = 0; i < nd; ++i) {
          const int d = lane + 32 * i;
          if (d < D) po[d] = acc[i] * inv;
        }
        if (lane == 0) p.part_lse[slot * p.Hq + hq] = lse;
      }
    };
    int cb = b0;
    for (int64_t fp = s; fp < e; ++fp) {
      while (prefix[cb + 1] <= fp) ++cb;
      if (cb != cur_b) {
        if (cur_b >= 0) finish(cur_b, fp);
        cur_b = cb;
        cur_len = eff_len(p, cb);
        seg_first = fp;
        const T* qr = reinterpret_cast<const T*>(p.q) + static_cast<int64_t>(cb) * p.q_sb +
                      static_cast<int64_t>(hq) * p.q_sh;
        for (int i = 0; i < 8; ++i) {
          const int d = lane + 32 * i;
          qv[i] = (i < nd && d < D) ? Elem<T>::to_f(qr[d]) : 0.f;
          acc[i] = 0.f;
        }
        m = -INFINITY;
        l = 0.f;
      }
      const int j = static_cast<int>(fp - prefix[cb]);
      const int page = __ldg(p.bt + static_cast<int64_t>(cb) * p.bt_sb + j);
      const int rows = min(kPage, cur_len - j * kPage);
      for (int t = 0; t < rows; ++t) {
        const int64_t off = static_cast<int64_t>(page) * p.page_stride +
                            (static_cast<int64_t>(t) * p.Hkv + h) * D;
        float dot = 0.f;
        for (int i = 0; i < nd; ++i) {
          const int d = lane + 32 * i;
          if (d < D) dot += qv[i] * Elem<T>::to_f(kg[off + d]);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
        const float sc = dot * p.scale;
        const float mn = fmaxf(m, sc);
        const float alpha = expf(m - mn);
        const float pr = expf(sc - mn);
        l = l * alpha + pr;
        for (int i = 0; i < nd; ++i) {
          const int d = lane + 32 * i;
          const float vv = (d < D) ? Elem<T>::to_f(vg[off + d]) : 0.f;
          acc[i] = acc[i] * alpha + pr * vv;
        }
        m = mn;
      }
    }
    if (cur_b >= 0) finish(cur_b, e);
  }
}

// ---------------------------------------------------------------------------
// LSE merge of partials: rows of `parts` at stride part_stride (elements of
// one part); out row r = sum_i exp(lse_i - M) o_i / sum_i exp(lse_i - M).
// ---------------------------------------------------------------------------
template <typename T>
__device__ void lse_merge_row(const float* part_o, const float* part_lse, int64_t part_stride_o,
                              int64_t part_stride_lse, int nparts, int D, T* out_row,
                              float* lse_out, int tid, int nthr) {
  float M = -INFINITY;
  for (int i = 0; i < nparts; ++i) M = fmaxf(M, part_lse[i * part_stride_lse]);
  if (M == -INFINITY) {
    for (int d = tid; d < D; d += nthr) out_row[d] = Elem<T>::from_f(__int_as_float(0x7fc00000));
    if (lse_out != nullptr && tid == 0) *lse_out = -INFINITY;
    return;
  }
  float W = 0.f;
  for (int i = 0; i < nparts; ++i) W += expf(part_lse[i * part_stride_lse] - M);
  const float invW = 1.f / W;
  for (int d = tid; d < D; d += nthr) {
    float a = 0.f;
    for (int i = 0; i < nparts; ++i) {
      const float w = expf(part_lse[i * part_stride_lse] - M);
      if (w > 0.f) a += w * part_o[i * part_stride_o + d];
    }
    out_row[d] = Elem<T>::from_f(a * invW);
  }
  if (lse_out != nullptr && tid == 0) *lse_out = M + logf(W);
}

// Combine of split requests.  CTA (b, q-head, 32 head_dim columns), 8 warps.
// The CTAs that own pages of request b are c_lo..c_hi; when every CTA range is
// non-empty (T >= G) their slots are simply c + b, otherwise (few pages) the
// empty ranges are skipped with a short serial scan.  Requests without pages
// get NaN rows (the reference's 0/0); requests owned by a single CTA were
// finished by the decode kernel (unless partials_only).
constexpr int kMaxSlotsPerReq = 1024;  // >= 2 * SM count
constexpr int kCombWarps = 8;

// Merges the partials of request b (pages first..last-1 of the flattened list),
// q-head hq, columns d0 + lane.  Call with the whole CTA; on return warp 0 holds
// o (its lane's column) and lse of the merged row.  The weights exp(lse_i - M)
// are formed once in shared memory (M and their sum by block reductions); warp
// w then accumulates slots w, w+8, ... over its lane's column (coalesced rows
// of the partial buffer), and the 8 warp sums are added in a fixed order.
// (Measured against an online log-sum-exp that skips the max pass: this form
// was faster for the many short combines of a large batch and equal for one
// long request.)
__device__ void combine_partials(const DecodeParams& p, int G, int b, int hq, int d0, int64_t first,
                                 int64_t last, float& o, float& lse) {
  __shared__ int s_slot[kMaxSlotsPerReq];
  __shared__ float s_w[kMaxSlotsPerReq];
  __shared__ float s_red[kCombWarps];
  __shared__ float s_acc[kCombWarps][32];
  __shared__ int s_n;
  const int64_t T_ = p.g_prefix[p.B];
  const int c_lo = owner_of_page(first, T_, G), c_hi = owner_of_page(last - 1, T_, G);
  const bool dense = T_ >= G;  // every CTA owns >= 1 page
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (!dense && threadIdx.x == 0) {
    int n = 0;
    int64_t start = range_start(c_lo, T_, G);
    for (int c = c_lo; c <= c_hi && n < kMaxSlotsPerReq; ++c) {
      const int64_t next = range_start(c + 1, T_, G);
      if (next > start) s_slot[n++] = c + b;
      start = next;
    }
    s_n = n;
  }
  __syncthreads();
  const int n = dense ? min(c_hi - c_lo + 1, kMaxSlotsPerReq) : s_n;
  auto slot = [&](int i) { return dense ? (c_lo + i + b) : s_slot[i]; };
  float M = -INFINITY;
  for (int i = threadIdx.x; i < n; i += blockDim.x) M = fmaxf(M, p.part_lse[static_cast<int64_t>(slot(i)) * p.Hq + hq]);
  for (int o2 = 16; o2 > 0; o2 >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o2));
  if (lane == 0) s_red[warp] = M;
  __syncthreads();
  M = s_red[0];
  for (int w = 1; w < kCombWarps; ++w) M = fmaxf(M, s_red[w]);
  __syncthreads();
  float W = 0.f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float w = expf(p.part_lse[static_cast<int64_t>(slot(i)) * p.Hq + hq] - M);
    s_w[i] = w;
    W += w;
  }
  for (int o2 = 16; o2 > 0; o2 >>= 1) W += __shfl_xor_sync(0xffffffffu, W, o2);
  if (lane == 0) s_red[warp] = W;
  __syncthreads();
  W = 0.f;
  for (int w = 0; w < kCombWarps; ++w) W += s_red[w];
  const int d = d0 + lane;
  float acc = 0.f;
#pragma unroll 8
  for (int i = warp; i < n; i += kCombWarps) {
    const float* po = p.part_o + (static_cast<int64_t>(slot(i)) * p.Hq + hq) * p.D;
    if (d < p.D) acc += s_w[i] * po[d];
  }
  s_acc[warp][lane] = acc;
  __syncthreads();
  if (warp == 0) {
    float a = 0.f;
    for (int w = 0; w < kCombWarps; ++w) a += s_acc[w][lane];
    o = a / W;
    lse = M + logf(W);
  }
}

template <typename T>
__global__ void __launch_bounds__(kCombWarps * 32) page16_decode_combine_kernel(DecodeParams p, int G) {
  // launched as a programmatic dependent of the decode kernel: wait until that grid has
  // completed and its partials are visible (a no-op for an ordinary launch)
  pdl_wait();
  // a programmatic dependent of this grid may become resident now; it waits for this
  // grid's completion itself
  asm volatile("griddepcontrol.launch_dependents;" :::);
  const int b = blockIdx.x, hq = blockIdx.y;
  const int d0 = blockIdx.z * 32;  // this CTA's 32 head_dim columns
  const int D = p.D;
  if (d0 >= D) return;
  const int64_t T_ = p.g_prefix[p.B];
  const int64_t first = p.g_prefix[b], last = p.g_prefix[b + 1];
  T* ob = reinterpret_cast<T*>(p.out) + (static_cast<int64_t>(b) * p.Hq + hq) * D;
  float* lse_dst = (p.lse_out && blockIdx.z == 0) ? p.lse_out + static_cast<int64_t>(b) * p.Hq + hq : nullptr;
  if (last == first) {
    for (int d = d0 + threadIdx.x; d < min(D, d0 + 32); d += blockDim.x) ob[d] = Elem<T>::from_f(__int_as_float(0x7fc00000));
    if (lse_dst != nullptr && threadIdx.x == 0) *lse_dst = -INFINITY;
    return;
  }
  if (!p.partials_only && owner_of_page(first, T_, G) == owner_of_page(last - 1, T_, G)) return;
  float o = 0.f, lse = 0.f;
  combine_partials(p, G, b, hq, d0, first, last, o, lse);
  if (threadIdx.x < 32) {
    if (d0 + threadIdx.x < D) ob[d0 + threadIdx.x] = Elem<T>::from_f(o);
    if (lse_dst != nullptr && threadIdx.x == 0) *lse_dst = lse;
  }
}

template <typename T>
__global__ void lse_combine_kernel(const float* part_o, const float* part_lse, void* out,
                                   float* lse_out, int nparts, int rows, int D) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  const int r = blockIdx.x * nw + warp;
  if (r >= rows) return;
  lse_merge_row<T>(part_o + static_cast<int64_t>(r) * D, part_lse + r, static_cast<int64_t>(rows) * D,
                   rows, nparts, D, reinterpret_cast<T*>(out) + static_cast<int64_t>(r) * D,
                   lse_out ? lse_out + r : nullptr, lane, 32);
}

// ---------------------------------------------------------------------------
// Split-KV decode of sequences whose pages are split across GPUs: the decode
// grid (partials_only) leaves one fp32 partial per CTA of every request, and
// this kernel - a programmatic dependent launch of that grid - does the rest of
// the layer, one CTA of kCombWarps warps per (row r = (request b, q-head),
// 32 head_dim columns):
//   1. local combine: the row's CTA partials (fp32, workspace slots) merged by
//      log-sum-exp (combine_partials) into this rank's (o, lse) for the CTA's
//      columns, kept in fp32;
//   2. exchange: those columns of (o, lse) stored into every peer's exchange
//      buffer as words that carry the call number (peer_words.cuh), over NVLink
//      (the lse word by the column-0 CTA);
//   3. merge: the peers' lse words and the CTA's data words for this row polled
//      from this rank's own buffer (bounded waits) and merged with the own
//      (o, lse) in fp32, written once as TO (and lse_out).
// So no partial is rounded to a 16-bit type before the final merge, and a layer
// is two launches (decode, this) instead of three.  With world == 1 steps 2 and
// 3 reduce to the local combine.  A wait that runs out sets *status = 1 and
// writes a NaN row.
// ---------------------------------------------------------------------------
struct PeerSet {
  uint4* bufs[peer::kMaxRanks];
  int* status;
  int rank, world;
  uint32_t max_polls;
};

template <typename T, typename TO>
__global__ void __launch_bounds__(kCombWarps * 32) split_kv_p2p_kernel(DecodeParams p, int G,
                                                                       const __grid_constant__ PeerSet ps) {
  __shared__ float s_o[32];
  __shared__ float s_lse;
  __shared__ float s_lq[peer::kMaxRanks];
  pdl_wait();  // the decode grid's partials and prefix are complete and visible
  asm volatile("griddepcontrol.launch_dependents;" :::);
  const int r = blockIdx.x, rows = p.B * p.Hq;
  const int b = r / p.Hq, hq = r % p.Hq;
  const int D = p.D, tid = threadIdx.x;
  const int d0 = blockIdx.y * 32;
  const int64_t first = p.g_prefix[b], last = p.g_prefix[b + 1];
  // ---- 1. local combine of the CTA partials of request b (this CTA's columns) ----
  if (last > first) {
    float o = 0.f, lse = 0.f;
    combine_partials(p, G, b, hq, d0, first, last, o, lse);
    if (tid < 32) s_o[tid] = o;
    if (tid == 0) s_lse = lse;
  } else {
    if (tid < 32) s_o[tid] = 0.f;
    if (tid == 0) s_lse = -INFINITY;
  }
  __syncthreads();
  const float lse_mine = s_lse;
  // ---- 2. exchange: words [j0, j1) of the row (+ the lse word from the column-0 CTA) ----
  const int H = D / 2, j0 = d0 / 2, j1 = min(H, j0 + 16);
  const int nw = (j1 - j0) + (blockIdx.y == 0 ? 1 : 0);
  uint32_t epoch = 0;
  int par = 0;
  if (ps.world > 1) {
    uint4* own = ps.bufs[ps.rank];
    epoch = *peer::epoch_ptr(own, ps.world, rows, D) + 1u;
    par = static_cast<int>(epoch & 1u);
    for (int e = tid; e < (ps.world - 1) * nw; e += blockDim.x) {
      const int i = e / nw, k = e % nw;
      const int pr = (ps.rank + 1 + i) % ps.world;
      const int j = (k < j1 - j0) ? j0 + k : H;
      const float x0 = j < H ? s_o[2 * (j - j0)] : lse_mine;
      const float x1 = j < H ? s_o[2 * (j - j0) + 1] : 0.f;
      peer::st_word(peer::row_ptr(ps.bufs[pr], ps.world, rows, D, par, ps.rank, r) + j, x0, x1, epoch);
    }
  }
  // ---- 3. merge ----
  const uint64_t t0 = peer::now_ns();
  uint32_t polls = 0;
  bool ok = true;
  if (tid < peer::kMaxRanks) {
    float lq = -INFINITY;
    if (tid == ps.rank) {
      lq = lse_mine;
    } else if (tid < ps.world) {
      float unused;
      ok = peer::wait_word(peer::row_ptr(ps.bufs[ps.rank], ps.world, rows, D, par, tid, r) + H, epoch, polls,
                           ps.max_polls, t0, lq, unused);
    }
    s_lq[tid] = lq;
  }
  const bool failed_lse = __syncthreads_or(!ok);
  float Mg = -INFINITY;
  for (int q = 0; q < ps.world; ++q) Mg = fmaxf(Mg, s_lq[q]);
  float v0 = 0.f, v1 = 0.f, Wg = 0.f;
  const int j = j0 + tid;
  if (!failed_lse && Mg != -INFINITY && tid < 16) {
    for (int q = 0; q < ps.world; ++q) {
      const float wq = expf(s_lq[q] - Mg);
      Wg += wq;
      if (!(wq > 0.f) || j >= j1) continue;
      float x0, x1;
      if (q == ps.rank) {
        x0 = s_o[2 * tid];
        x1 = s_o[2 * tid + 1];
      } else if (!peer::wait_word(peer::row_ptr(ps.bufs[ps.rank], ps.world, rows, D, par, q, r) + j, epoch,
                                  polls, ps.max_polls, t0, x0, x1)) {
        ok = false;
        x0 = x1 = 0.f;
      }
      v0 += wq * x0;
      v1 += wq * x1;
    }
  }
  const bool failed = __syncthreads_or(!ok);
  TO* ob = reinterpret_cast<TO*>(p.out) + static_cast<int64_t>(r) * D;
  const float nan = __int_as_float(0x7fc00000);
  if (failed || Mg == -INFINITY) {  // a wait ran out, or no rank had keys for this row (the reference's 0/0)
    for (int d = d0 + tid; d < min(D, d0 + 32); d += blockDim.x) ob[d] = Elem<TO>::from_f(nan);
    if (tid == 0 && blockIdx.y == 0 && p.lse_out != nullptr) p.lse_out[r] = failed ? nan : -INFINITY;
    if (tid == 0 && failed) atomicExch(ps.status, 1);
  } else {
    if (tid < 16 && j < j1) {
      const float invg = 1.f / Wg;
      ob[2 * j] = Elem<TO>::from_f(v0 * invg);
      ob[2 * j + 1] = Elem<TO>::from_f(v1 * invg);
    }
    if (tid == 0 && blockIdx.y == 0 && p.lse_out != nullptr) {
      float W = 0.f;
      for (int q = 0; q < ps.world; ++q) W += expf(s_lq[q] - Mg);
      p.lse_out[r] = Mg + logf(W);
    }
  }
  if (ps.world > 1) {
    __syncthreads();
    if (tid == 0) peer::finish_call(ps.bufs[ps.rank], ps.world, rows, D, epoch);
  }
}

// ---------------------------------------------------------------------------
// Decode-token append.

// Append for the generic decode path: the new token goes to position len-1 (lengths include it).
template <typename T>
__global__ void decode_append_len_kernel(DecodeParams p) {
  const int b = blockIdx.x;
  const int len = p.lens[b];
  if (len <= 0 || len > p.max_blocks * kPage) return;
  const int pos = len - 1;
  const int page = p.bt[static_cast<int64_t>(b) * p.bt_sb + pos / kPage];
  const int64_t dst = static_cast<int64_t>(page) * p.page_stride + static_cast<int64_t>(pos % kPage) * p.Hkv * p.D;
  const int64_t src = static_cast<int64_t>(b) * p.new_sb;
  T* kc = const_cast<T*>(reinterpret_cast<const T*>(p.k));
  T* vc = const_cast<T*>(reinterpret_cast<const T*>(p.v));
  for (int i = threadIdx.x; i < p.Hkv * p.D; i += blockDim.x) {
    kc[dst + i] = reinterpret_cast<const T*>(p.k_new)[src + i];
    vc[dst + i] = reinterpret_cast<const T*>(p.v_new)[src + i];
  }
}
// ---------------------------------------------------------------------------
template <typename T>
__global__ void decode_append_kernel(const T* k_new, const T* v_new, T* k_cache, T* v_cache,
                                     const int32_t* bt, const int32_t* old_lens, int Hkv, int D,
                                     int max_blocks, int64_t new_sb, int64_t page_stride,
                                     int64_t bt_sb) {
  const int b = blockIdx.x;
  const int old = old_lens[b];
  if (old < 0 || old >= max_blocks * kPage) return;
  const int page = bt[static_cast<int64_t>(b) * bt_sb + old / kPage];
  const int slot = old % kPage;
  const int64_t dst = static_cast<int64_t>(page) * page_stride + static_cast<int64_t>(slot) * Hkv * D;
  const int64_t src = static_cast<int64_t>(b) * new_sb;
  const int n = Hkv * D;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    k_cache[dst + i] = k_new[src + i];
    v_cache[dst + i] = v_new[src + i];
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

struct WsLayout {
  size_t prefix_off, lse_off, o_off, total;
};

WsLayout ws_layout(int batch, int Hq, int D) {
  const int64_t slots = 2LL * sm_count() + batch;
  WsLayout w;
  w.prefix_off = 0;
  w.lse_off = align_up(sizeof(int32_t) * (static_cast<size_t>(batch) + 1), 256);
  w.o_off = w.lse_off + align_up(sizeof(float) * slots * Hq, 256);
  w.total = w.o_off + align_up(sizeof(float) * slots * Hq * D, 256);
  return w;
}

// Raises the dynamic shared memory limit of `kernel` once per device; `done`
// is the caller's per-kernel flag array.
template <typename K>
bool set_smem(K kernel, size_t bytes, bool* done) {
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && done[dev]) return true;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(bytes)) != cudaSuccess)
    return false;
  if (dev >= 0 && dev < 64) done[dev] = true;
  return true;
}

// CTAs over the flattened page list: one per SM and KV-head group by default, or the
// caller's split count (at most 2 per SM: the workspace holds 2*SMs + B partial slots).
inline int decode_grid(const DecodeParams& p, int groups) {
  const int dflt = max(1, sm_count() / groups);
  if (p.num_splits <= 0) return dflt;
  return max(1, min(p.num_splits, 2 * sm_count() / groups));
}

template <typename T, int D, int NW, int NS>
int launch_mma(DecodeParams& p, cudaStream_t st, bool combine) {
  const int groups = (p.Hkv + NW - 1) / NW;
  const int G = decode_grid(p, groups);
  const size_t smem = static_cast<size_t>(NW) * NS * 2 * 16 * D * 2 + sizeof(int) * (p.B + 1);
  auto kern = page16_decode_mma_kernel<T, D, NW, NS>;
  static bool done[64] = {false};
  if (!set_smem(kern, NW * NS * 2 * 16 * D * 2 + sizeof(int) * 4097, done)) {
    set_error("page16_native_launch:smem_attr");
    return BPKV_ERR_CUDA;
  }
  // an ordinary launch (measured: as a programmatic dependent of the previous layer's
  // combine it gained nothing on the batched decode)
  kern<<<dim3(G, groups), NW * 32, smem, st>>>(p);
  if (!combine) BPKV_RETURN_LAUNCH("page16_native_launch");
  // the combine overlaps its launch with the decode grid's tail (programmatic dependent launch)
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.B, p.Hq, (p.D + 31) / 32);
  cfg.blockDim = dim3(kCombWarps * 32);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t le = cudaLaunchKernelEx(&cfg, page16_decode_combine_kernel<T>, p, G);
  if (le != cudaSuccess) {
    set_error("page16_native_launch:%s", cudaGetErrorString(le));
    return BPKV_ERR_CUDA;
  }
  BPKV_RETURN_LAUNCH("page16_native_launch");
}

template <typename T>
__global__ void decode_append_kernel(const T* k_new, const T* v_new, T* k_cache, T* v_cache,
                                     const int32_t* bt, const int32_t* old_lens, int Hkv, int D,
                                     int max_blocks, int64_t new_sb, int64_t page_stride,
                                     int64_t bt_sb);
template <typename T>
__global__ void decode_append_len_kernel(DecodeParams p);

template <typename T>
int launch_generic(DecodeParams& p, cudaStream_t st, bool combine) {
  constexpr int NW = 8;
  if (p.k_new != nullptr) decode_append_len_kernel<T><<<p.B, 256, 0, st>>>(p);  // append, then decode
  const int G = decode_grid(p, 1);
  const size_t smem = sizeof(int) * (p.B + 1);
  auto kern = page16_decode_generic_kernel<T, NW>;
  static bool done[64] = {false};
  if (smem > 48 * 1024 && !set_smem(kern, sizeof(int) * (16384 + 1), done)) {
    set_error("page16_native_launch:smem_attr");
    return BPKV_ERR_CUDA;
  }
  kern<<<G, NW * 32, smem, st>>>(p);
  if (!combine) BPKV_RETURN_LAUNCH("page16_native_launch");
  page16_decode_combine_kernel<T><<<dim3(p.B, p.Hq, (p.D + 31) / 32), kCombWarps * 32, 0, st>>>(p, G);
  BPKV_RETURN_LAUNCH("page16_native_launch");
}

// Decode grid G of the launch that dispatch() makes for these parameters.
inline int dispatch_grid(const DecodeParams& p, bool fast_ok) {
  if (fast_ok && p.D == 256) return decode_grid(p, (p.Hkv + 3) / 4);
  if (fast_ok) return decode_grid(p, (p.Hkv + 7) / 8);
  return decode_grid(p, 1);
}

template <typename T>
int dispatch(DecodeParams& p, cudaStream_t st, bool fast_ok, bool combine = true) {
  if constexpr (!std::is_same<T, float>::value) {
    if (fast_ok) {
      if (p.D == 128) return launch_mma<T, 128, 8, 3>(p, st, combine);
      if (p.D == 64) return launch_mma<T, 64, 8, 6>(p, st, combine);
      if (p.D == 256) return launch_mma<T, 256, 4, 3>(p, st, combine);
    }
  }
  return launch_generic<T>(p, st, combine);
}

}  // namespace
}  // namespace bpkv

using namespace bpkv;

extern "C" BPKV_API size_t bpkv_page16_decode_workspace_size(int batch, int num_q_heads, int num_kv_heads,
                                                    int head_dim, int dtype) {
  (void)num_kv_heads;
  (void)dtype;
  if (batch <= 0 || num_q_heads <= 0 || head_dim <= 0) return 0;
  return ws_layout(batch, num_q_heads, head_dim).total;
}

// Validates the arguments and fills the kernel parameters (shared by every decode entry point).
static int fill_decode_params(DecodeParams& p, bool& fast_ok, const void* q, const void* k_cache,
                              const void* v_cache, const int32_t* block_table, const int32_t* cache_seqlens,
                              void* out, float* lse_out, int batch, int num_q_heads, int num_kv_heads,
                              int head_dim, int max_blocks, int64_t q_stride_b, int64_t q_stride_h,
                              int64_t page_stride, int64_t bt_stride_b, float softmax_scale, int dtype,
                              void* workspace, size_t workspace_bytes, const void* k_new, const void* v_new,
                              int64_t new_stride_b) {
  BPKV_CHECK_ARG(batch > 0 && num_q_heads > 0 && head_dim > 0, "page16_native_shape_unsupported:empty");
  BPKV_CHECK_ARG(num_kv_heads > 0 && num_q_heads % num_kv_heads == 0, "page16_native_shape_unsupported:gqa");
  BPKV_CHECK_ARG(head_dim <= 256, "page16_native_shape_unsupported:head_dim_%d", head_dim);
  BPKV_CHECK_ARG(max_blocks >= 0, "page16_native_shape_unsupported:block_table_rank");
  BPKV_CHECK_ARG(batch <= 16384, "page16_native_shape_unsupported:batch_%d", batch);
  BPKV_CHECK_ARG(dtype == BPKV_F32 || dtype == BPKV_F16 || dtype == BPKV_BF16,
                 "page16_native_shape_unsupported:dtype_%d", dtype);
  BPKV_CHECK_ARG(q && k_cache && v_cache && cache_seqlens && out, "page16_native_shape_unsupported:null_pointer");
  BPKV_CHECK_ARG(max_blocks == 0 || block_table != nullptr, "page16_native_shape_unsupported:null_pointer");
  const WsLayout w = ws_layout(batch, num_q_heads, head_dim);
  if (workspace == nullptr || workspace_bytes < w.total) {
    set_error("page16_native_workspace:need_%zu_bytes", w.total);
    return BPKV_ERR_WORKSPACE;
  }
  memset(&p, 0, sizeof(p));
  p.q = q;
  p.k = k_cache;
  p.v = v_cache;
  p.bt = block_table;
  p.lens = cache_seqlens;
  p.out = out;
  p.lse_out = lse_out;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  p.g_prefix = reinterpret_cast<int32_t*>(ws + w.prefix_off);
  p.part_lse = reinterpret_cast<float*>(ws + w.lse_off);
  p.part_o = reinterpret_cast<float*>(ws + w.o_off);
  p.B = batch;
  p.Hq = num_q_heads;
  p.Hkv = num_kv_heads;
  p.D = head_dim;
  p.max_blocks = max_blocks;
  p.n_rep = num_q_heads / num_kv_heads;
  p.q_sb = q_stride_b;
  p.q_sh = q_stride_h;
  p.page_stride = page_stride;
  p.bt_sb = bt_stride_b;
  p.scale = softmax_scale;
  p.scale_log2 = softmax_scale * 1.4426950408889634f;
  p.k_new = k_new;
  p.v_new = v_new;
  p.new_sb = new_stride_b;
  fast_ok = dtype != BPKV_F32 && (head_dim == 64 || head_dim == 128 || head_dim == 256) && p.n_rep <= 16 &&
            batch <= 4096 && aligned16(q) && aligned16(k_cache) && aligned16(v_cache) && aligned16(out) &&
            (q_stride_b % 8 == 0) && (q_stride_h % 8 == 0) && (page_stride % 8 == 0) &&
            (k_new == nullptr || (aligned16(k_new) && aligned16(v_new) && new_stride_b % 8 == 0));
  return BPKV_OK;
}

static int page16_decode_impl(const void* q, const void* k_cache, const void* v_cache,
                              const int32_t* block_table, const int32_t* cache_seqlens, void* out,
                              float* lse_out, int batch, int num_q_heads, int num_kv_heads, int head_dim,
                              int max_blocks, int64_t q_stride_b, int64_t q_stride_h, int64_t page_stride,
                              int64_t bt_stride_b, float softmax_scale, int dtype, void* workspace,
                              size_t workspace_bytes, void* stream, const void* k_new, const void* v_new,
                              int64_t new_stride_b) {
  clear_error();
  DecodeParams p;
  bool fast_ok = false;
  const int rc = fill_decode_params(p, fast_ok, q, k_cache, v_cache, block_table, cache_seqlens, out, lse_out,
                                    batch, num_q_heads, num_kv_heads, head_dim, max_blocks, q_stride_b,
                                    q_stride_h, page_stride, bt_stride_b, softmax_scale, dtype, workspace,
                                    workspace_bytes, k_new, v_new, new_stride_b);
  if (rc != BPKV_OK) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == BPKV_BF16) return dispatch<__nv_bfloat16>(p, st, fast_ok);
  if (dtype == BPKV_F16) return dispatch<__half>(p, st, fast_ok);
  return dispatch<float>(p, st, false);
}

extern "C" BPKV_API int bpkv_page16_decode(const void* q, const void* k_cache, const void* v_cache,
                                           const int32_t* block_table, const int32_t* cache_seqlens, void* out,
                                           float* lse_out, int batch, int num_q_heads, int num_kv_heads,
                                           int head_dim, int max_blocks, int64_t q_stride_b, int64_t q_stride_h,
                                           int64_t page_stride, int64_t bt_stride_b, float softmax_scale, int dtype,
                                           void* workspace, size_t workspace_bytes, void* stream) {
  return page16_decode_impl(q, k_cache, v_cache, block_table, cache_seqlens, out, lse_out, batch, num_q_heads,
                            num_kv_heads, head_dim, max_blocks, q_stride_b, q_stride_h, page_stride, bt_stride_b,
                            softmax_scale, dtype, workspace, workspace_bytes, stream, nullptr, nullptr, 0);
}

extern "C" BPKV_API int bpkv_page16_decode_append(const void* q, const void* k_new, const void* v_new,
                                                  int64_t new_stride_b, void* k_cache, void* v_cache,
                                                  const int32_t* block_table, const int32_t* cache_seqlens,
                                                  void* out, float* lse_out, int batch, int num_q_heads,
                                                  int num_kv_heads, int head_dim, int max_blocks, int64_t q_stride_b,
                                                  int64_t q_stride_h, int64_t page_stride, int64_t bt_stride_b,
                                                  float softmax_scale, int dtype, void* workspace,
                                                  size_t workspace_bytes, void* stream) {
  if (k_new == nullptr || v_new == nullptr) {
    clear_error();
    set_error("page16_native_shape_unsupported:null_new_token");
    return BPKV_ERR_SHAPE;
  }
  return page16_decode_impl(q, k_cache, v_cache, block_table, cache_seqlens, out, lse_out, batch, num_q_heads,
                            num_kv_heads, head_dim, max_blocks, q_stride_b, q_stride_h, page_stride, bt_stride_b,
                            softmax_scale, dtype, workspace, workspace_bytes, stream, k_new, v_new, new_stride_b);
}

extern "C" BPKV_API int bpkv_lse_combine(const float* part_out, const float* part_lse, void* out,
                                float* lse_out, int num_parts, int rows, int head_dim,
                                int out_dtype, void* stream) {
  clear_error();
  BPKV_CHECK_ARG(num_parts > 0 && rows >= 0 && head_dim > 0, "lse_combine_shape_unsupported:empty");
  BPKV_CHECK_ARG(part_out && part_lse && out, "lse_combine_shape_unsupported:null_pointer");
  if (rows == 0) return BPKV_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int nw = 8;
  const int grid = (rows + nw - 1) / nw;
  if (out_dtype == BPKV_F32)
    lse_combine_kernel<float><<<grid, nw * 32, 0, st>>>(part_out, part_lse, out, lse_out, num_parts, rows, head_dim);
  else if (out_dtype == BPKV_F16)
    lse_combine_kernel<__half><<<grid, nw * 32, 0, st>>>(part_out, part_lse, out, lse_out, num_parts, rows, head_dim);
  else if (out_dtype == BPKV_BF16)
    lse_combine_kernel<__nv_bfloat16><<<grid, nw * 32, 0, st>>>(part_out, part_lse, out, lse_out, num_parts, rows, head_dim);
  else
    BPKV_CHECK_ARG(false, "lse_combine_shape_unsupported:dtype_%d", out_dtype);
  BPKV_RETURN_LAUNCH("lse_combine_launch");
}

extern "C" BPKV_API int bpkv_decode_append(const void* k_new, const void* v_new, void* k_cache, void* v_cache,
                                  const int32_t* block_table, const int32_t* old_lens, int batch,
                                  int num_kv_heads, int head_dim, int max_blocks,
                                  int64_t new_stride_b, int64_t page_stride, int64_t bt_stride_b,
                                  int dtype, void* stream) {
  clear_error();
  BPKV_CHECK_ARG(batch >= 0 && num_kv_heads > 0 && head_dim > 0 && max_blocks >= 0,
                 "decode_append_shape_unsupported:empty");
  if (batch == 0 || max_blocks == 0) return BPKV_OK;
  BPKV_CHECK_ARG(k_new && v_new && k_cache && v_cache && block_table && old_lens,
                 "decode_append_shape_unsupported:null_pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int thr = 256;
#define BPKV_APPEND(TY)                                                                     \
  decode_append_kernel<TY><<<batch, thr, 0, st>>>(                                          \
      static_cast<const TY*>(k_new), static_cast<const TY*>(v_new), static_cast<TY*>(k_cache), \
      static_cast<TY*>(v_cache), block_table, old_lens, num_kv_heads, head_dim, max_blocks,   \
      new_stride_b, page_stride, bt_stride_b)
  if (dtype == BPKV_F32) BPKV_APPEND(float);
  else if (dtype == BPKV_F16) BPKV_APPEND(__half);
  else if (dtype == BPKV_BF16) BPKV_APPEND(__nv_bfloat16);
  else BPKV_CHECK_ARG(false, "decode_append_shape_unsupported:dtype_%d", dtype);
#undef BPKV_APPEND
  BPKV_RETURN_LAUNCH("decode_append_launch");
}

// ---------------------------------------------------------------------------
// Allocation-free variant of bpkv_page16_decode.
//
// Some callers cannot allocate device memory at decode time: an engine that
// has handed (nearly) all of HBM to the paged pool up front, a host written in
// another language that reaches this library through a plain C FFI and owns no
// device allocator, or a latency-critical loop that must not hit cudaMalloc's
// implicit device synchronisation.  For them the split-KV scratch (request
// page prefix, per-slot partial outputs and log-sum-exps) lives in one
// file-scope device array of fixed size, kNoAllocScratchBytes, which every GPU
// that loads this library holds until the process exits.
//
// The array's host-side name is not a device address, so the address is
// looked up with cudaGetSymbolAddress once per device (with that device
// current) on the first call made on that device; make that first call before
// any stream capture.  Every call shares the same array: calls whose kernels
// overlap on the GPU (different streams, or different host threads without
// ordering) race on it and must be serialised by the caller.  Nothing in it
// has to start at zero: each call writes every scratch byte it later reads.
// ---------------------------------------------------------------------------
namespace bpkv {
namespace {
constexpr size_t kNoAllocScratchBytes = 16u << 20;  // 16 MiB
__device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

void* noalloc_scratch_ptr(int* err) {
  static std::mutex mu;
  static void* ptrs[64] = {nullptr};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    *err = 1;
    return nullptr;
  }
  std::lock_guard<std::mutex> lk(mu);
  if (ptrs[dev] == nullptr) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) {
      set_error("page16_native_noalloc:cudaGetSymbolAddress: %s", cudaGetErrorString(e));
      *err = 2;
      return nullptr;
    }
    ptrs[dev] = p;
  }
  return ptrs[dev];
}
}  // namespace
}  // namespace bpkv

extern "C" BPKV_API size_t bpkv_page16_decode_noalloc_max_scratch(void) { return bpkv::kNoAllocScratchBytes; }

extern "C" BPKV_API int bpkv_page16_decode_noalloc(const void* q, const void* k_cache, const void* v_cache,
                                                   const int32_t* block_table, const int32_t* cache_seqlens,
                                                   void* out, float* lse_out, int batch, int num_q_heads,
                                                   int num_kv_heads, int head_dim, int max_blocks,
                                                   int64_t q_stride_b, int64_t q_stride_h, int64_t page_stride,
                                                   int64_t bt_stride_b, float softmax_scale, int dtype,
                                                   void* stream) {
  clear_error();
  BPKV_CHECK_ARG(batch > 0 && num_q_heads > 0 && head_dim > 0, "page16_native_shape_unsupported:empty");
  const size_t need = ws_layout(batch, num_q_heads, head_dim).total;
  if (need > kNoAllocScratchBytes) {
    set_error("page16_native_noalloc:scratch_need_%zu_bytes_exceeds_max_%zu", need, kNoAllocScratchBytes);
    return BPKV_ERR_WORKSPACE;
  }
  int err = 0;
  void* scratch = noalloc_scratch_ptr(&err);
  if (scratch == nullptr) {
    if (err == 1) set_error("page16_native_noalloc:no_current_device");
    return BPKV_ERR_CUDA;
  }
  return bpkv_page16_decode(q, k_cache, v_cache, block_table, cache_seqlens, out, lse_out, batch, num_q_heads,
                            num_kv_heads, head_dim, max_blocks, q_stride_b, q_stride_h, page_stride, bt_stride_b,
                            softmax_scale, dtype, scratch, kNoAllocScratchBytes, stream);
}

// ---------------------------------------------------------------------------
// Split-KV decode with the NVLink exchange fused into the combine.
// ---------------------------------------------------------------------------
extern "C" BPKV_API int bpkv_split_kv_decode_p2p(const void* q, const void* k_cache, const void* v_cache,
                                                 const int32_t* block_table, const int32_t* cache_seqlens,
                                                 void* out, float* lse_out, int batch, int num_q_heads,
                                                 int num_kv_heads, int head_dim, int max_blocks,
                                                 int64_t q_stride_b, int64_t q_stride_h, int64_t page_stride,
                                                 int64_t bt_stride_b, float softmax_scale, int dtype,
                                                 int out_dtype, void* workspace, size_t workspace_bytes,
                                                 int num_splits,
                                                 void* const* peer_bufs, int rank, int world, uint32_t max_polls,
                                                 int* status, void* stream) {
  clear_error();
  BPKV_CHECK_ARG(world >= 1 && world <= peer::kMaxRanks && rank >= 0 && rank < world,
                 "peer_exchange_shape:rank_%d_of_%d", rank, world);
  BPKV_CHECK_ARG(head_dim % 4 == 0, "peer_exchange_shape:head_dim_%d", head_dim);
  BPKV_CHECK_ARG(status != nullptr, "peer_exchange_shape:null_pointer");
  BPKV_CHECK_ARG(out_dtype == dtype || out_dtype == BPKV_F32, "peer_exchange_shape:out_dtype_%d", out_dtype);
  BPKV_CHECK_ARG(world == 1 || peer_bufs != nullptr, "peer_exchange_shape:null_pointer");
  PeerSet ps;
  memset(&ps, 0, sizeof(ps));
  for (int r = 0; r < world && world > 1; ++r) {
    BPKV_CHECK_ARG(peer_bufs[r] != nullptr && aligned16(peer_bufs[r]), "peer_exchange_shape:buffer_%d", r);
    ps.bufs[r] = static_cast<uint4*>(peer_bufs[r]);
  }
  ps.status = status;
  ps.rank = rank;
  ps.world = world;
  ps.max_polls = max_polls;
  DecodeParams p;
  bool fast_ok = false;
  const int rc = fill_decode_params(p, fast_ok, q, k_cache, v_cache, block_table, cache_seqlens, out, lse_out,
                                    batch, num_q_heads, num_kv_heads, head_dim, max_blocks, q_stride_b,
                                    q_stride_h, page_stride, bt_stride_b, softmax_scale, dtype, workspace,
                                    workspace_bytes, nullptr, nullptr, 0);
  if (rc != BPKV_OK) return rc;
  p.partials_only = 1;
  p.num_splits = num_splits;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int G = dispatch_grid(p, fast_ok);
  int drc;
  if (dtype == BPKV_BF16) drc = dispatch<__nv_bfloat16>(p, st, fast_ok, false);
  else if (dtype == BPKV_F16) drc = dispatch<__half>(p, st, fast_ok, false);
  else drc = dispatch<float>(p, st, false, false);
  if (drc != BPKV_OK) return drc;
  const dim3 grid(batch * num_q_heads, (head_dim + 31) / 32), block(kCombWarps * 32);
  const bool f32_out = out_dtype == BPKV_F32;
  cudaError_t le;
  if (dtype == BPKV_BF16)
    le = f32_out ? launch_pdl(split_kv_p2p_kernel<__nv_bfloat16, float>, grid, block, 0, st, p, G, ps)
                 : launch_pdl(split_kv_p2p_kernel<__nv_bfloat16, __nv_bfloat16>, grid, block, 0, st, p, G, ps);
  else if (dtype == BPKV_F16)
    le = f32_out ? launch_pdl(split_kv_p2p_kernel<__half, float>, grid, block, 0, st, p, G, ps)
                 : launch_pdl(split_kv_p2p_kernel<__half, __half>, grid, block, 0, st, p, G, ps);
  else
    le = launch_pdl(split_kv_p2p_kernel<float, float>, grid, block, 0, st, p, G, ps);
  if (le != cudaSuccess) {
    set_error("split_kv_decode_p2p_launch:%s", cudaGetErrorString(le));
    return BPKV_ERR_CUDA;
  }
  BPKV_RETURN_LAUNCH("split_kv_decode_p2p_launch");
}
