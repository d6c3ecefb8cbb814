// Paged chunked-prefill / varlen attention on the 5th-generation tensor cores
// (tcgen05.mma with TMEM accumulators), sm_100a, head_dim 128, bf16 / fp16.
//
// Same semantics as prefill.cu (causal, bottom-right aligned; K/V read from
// 16-token pages through the block table, or dense varlen).  Per CTA:
//   * two Q tiles (groups A and B) of 128 accumulator rows each; a row is one
//     (query token, query head) pair of the n_rep heads of one KV head, so a
//     GQA group shares every K/V tile, and both tiles share the K/V loads.
//   * K/V tiles of 128 tokens (8 pages) land in 2-deep shared-memory rings in
//     the 128-byte-swizzled layout of the UMMA descriptors ([64-column block]
//     [token][128 B], 16-B chunk ^= token & 7).  Paged K/V come by TMA
//     (cp.async.bulk.tensor, 4-D tensor map over the pool layer, one 16x64 box
//     per page and half of head_dim, issued by 16 lanes of the load warp) and
//     are tracked by transaction bytes on per-buffer mbarriers; dense varlen
//     K/V come by 16-byte cp.async that arrive on the same mbarriers.
//   * one warp issues every tcgen05.mma: S_g = Q_g K^T (M128 N128, Q and K in
//     shared memory) and O_g += P_g V (M128 N128, P_g from TMEM, V as an
//     MN-major operand) in the order PV_A(j) S_A(j+1) PV_B(j) S_B(j+1), so the
//     softmax of one group runs while the tensor pipe works for the other.
//   * softmax: 8 warps per group, 2 threads per row (64 columns each), online
//     softmax in exp2 with a lazily moved reference max (O is rescaled in TMEM
//     only when a row max grows by more than 2^8); 1 in 8 exponentials is
//     evaluated on the FMA pipe by a polynomial to relieve the MUFU unit.  P
//     is written over S in TMEM as bf16 hi + lo parts (fp16: one part), which
//     keeps ~16 mantissa bits of each probability for the P.V product; a tile
//     whose weights are all small against their rows' running sums (decided
//     per group and tile) goes as the hi part alone, one P.V MMA instead of two.
// All waits are bounded; on a timeout the CTA stops, writes NaN rows and
// still frees its TMEM.  No TMA multicast is used (the loads read this GPU's
// own pool only).
#include <cuda.h>

#include "common.cuh"
#include "f32x2.cuh"
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

#ifdef BPKV_TRACE
// Debug builds only (-DBPKV_TRACE): per-phase clock64 totals of CTA (0,0).
__device__ unsigned long long g_prefill_trace[32];
#define BPKV_TRACING (blockIdx.x == 0)
// consecutive checkpoints of thread 0: slot k accumulates the cycles since the previous mark
#define BPKV_MARK(slot)                                                                          \
  do {                                                                                           \
    const long long _n = clock64();                                                              \
    if (BPKV_TRACING && tid == 0) atomicAdd(&g_prefill_trace[slot], static_cast<unsigned long long>(_n - _tl)); \
    _tl = _n;                                                                                    \
  } while (0)
#define BPKV_MARK_MMA(slot)                                                                      \
  do {                                                                                           \
    const long long _n = clock64();                                                              \
    if (BPKV_TRACING && lane == 0) atomicAdd(&g_prefill_trace[slot], static_cast<unsigned long long>(_n - _tm)); \
    _tm = _n;                                                                                    \
  } while (0)
#else
#define BPKV_MARK_MMA(slot) \
  do {                      \
  } while (0)
#define BPKV_MARK(slot) \
  do {                  \
  } while (0)
#endif

namespace {

// An M=128 tcgen05.mma costs the same tensor-pipe time for any N <= 128 (measured:
// ~64 cycles per K=16 step), so K/V tiles are 128 tokens: S = Q K^T runs at N=128.
// Two 128-row Q tiles per CTA (groups A and B) share every K/V tile; each has its
// own softmax warps, so the softmax of one group overlaps the other group's MMAs.
constexpr int kD = 128, kBM = 128, kBN = 128, kDB = kD / 64;
constexpr int kGroups = 2, kRows = kGroups * kBM;  // accumulator rows per CTA
constexpr int kQBytes = kDB * kBM * 128;       // 32 KB per Q tile
constexpr int kKVBytes = kDB * kBN * 128;      // 32 KB per K or V tile
constexpr int kNK = 2;                         // K ring depth (K(j) is free once S_B(j) completed)
constexpr int kNV = 2;                         // V ring depth (V(j) is free once PV_B(j) completed)
constexpr int kSplit = 2;                      // softmax threads per accumulator row
constexpr int kGroupWarps = 4 * kSplit;        // softmax warps per group
constexpr int kSoftmaxWarps = kGroups * kGroupWarps;  // warps 0..15
constexpr int kLoadWarp = kSoftmaxWarps;       // warp 16: TMA / cp.async loads
constexpr int kMmaWarp = kSoftmaxWarps + 1;    // warp 17: tcgen05.mma issue
constexpr int kThreads = (kSoftmaxWarps + 2) * 32;
static_assert(kThreads == (kMmaWarp + 1) * 32, "the MMA-issue warp is the last warp");
constexpr int kMaxPagesSmem = 2048;            // block-table entries staged in shared memory
constexpr int kSmemBytes = kGroups * kQBytes + (kNK + kNV) * kKVBytes + 1024 /*align*/ + 256 + 4 * kMaxPagesSmem +
                            4 * kGroups * 2 * kSplit * kBM /*row-max exchange*/ + 4 * kGroups * kSplit * kBM /*row sums*/;
// TMEM: group g owns S_g [256g, 256g+128) and O_g [256g+128, 256g+256).  P_g (16-bit pairs)
// overwrites S_g in place, chunk by chunk: the probabilities of S columns [32c, 32c+32) (tokens
// 32c..32c+31) go to columns [32c, 32c+16) (hi parts) and [32c+16, 32c+32) (lo parts).
constexpr uint32_t kTmemCols = 512;
#ifndef BPKV_PREFILL_SPLIT_P
#define BPKV_PREFILL_SPLIT_P 1
#endif
// bf16 P as hi + lo parts (default: two P.V MMAs per K step, ~16 mantissa bits per
// probability) or, with -DBPKV_PREFILL_SPLIT_P=0, as one bf16 part.  Measured at config-5
// shapes the single part runs at 1.3x the throughput, but one bf16 rounding of a weight
// costs up to 2^-9 relative: rows with few keys or one dominant key then miss the 2e-3
// max-abs bar (errors up to ~2^-9 |v|), as flash-attn's bf16 P does.
constexpr bool kSplitPBf16 = BPKV_PREFILL_SPLIT_P != 0;
#ifndef BPKV_PREFILL_LO_LOG2
#define BPKV_PREFILL_LO_LOG2 8
#endif
// a tile skips the lo part when every weight in it is <= 2^-kLoLog2 of its row's running sum
constexpr float kLoLog2 = BPKV_PREFILL_LO_LOG2;
constexpr float kRescaleThreshold = 8.0f;      // log2 units: P <= 256 between rescales

struct __align__(64) TcKernelArgs {
  CUtensorMap tmap_k;  // paged only
  CUtensorMap tmap_v;
  PrefillTcParams p;
};

__device__ __forceinline__ uint32_t sw_off(int row, int chunk) {  // chunk 0..7 inside a 128-B row
  return static_cast<uint32_t>(row * 128 + ((chunk ^ (row & 7)) << 4));
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap* map, int c0, int c1, int c2, int c3,
                                            uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], "
      "[%6];\n" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(bar)
      : "memory");
}
// Arrive on `bar` once all of this thread's prior cp.async copies have landed.
__device__ __forceinline__ void cp_async_arrive(uint32_t bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];\n" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};\n"
      "tcgen05.wait::st.sync.aligned;\n" ::"r"(taddr),
      "f"(v[0]), "f"(v[1]), "f"(v[2]), "f"(v[3]), "f"(v[4]), "f"(v[5]), "f"(v[6]), "f"(v[7]), "f"(v[8]), "f"(v[9]),
      "f"(v[10]), "f"(v[11]), "f"(v[12]), "f"(v[13]), "f"(v[14]), "f"(v[15]), "f"(v[16]), "f"(v[17]), "f"(v[18]),
      "f"(v[19]), "f"(v[20]), "f"(v[21]), "f"(v[22]), "f"(v[23]), "f"(v[24]), "f"(v[25]), "f"(v[26]), "f"(v[27]),
      "f"(v[28]), "f"(v[29]), "f"(v[30]), "f"(v[31])
      : "memory");
}

#ifndef BPKV_PREFILL_EMU
#define BPKV_PREFILL_EMU 8
#endif
constexpr int kEmuStride = BPKV_PREFILL_EMU;  // every kEmuStride-th exponential pair goes to the FMA pipe

constexpr int kMaxRanked = 512;  // q-tile items ranked per CTA (n^2 / kThreads compares)

// K/V tiles a (request, q-tile) item iterates over (-1: item past the request's queries)
__device__ __forceinline__ int item_tiles(const PrefillTcParams& p, int i) {
  const int b = i / p.tiles_per_req, qt = i % p.tiles_per_req;
  const int q0 = __ldg(p.cu_q + b), nq = __ldg(p.cu_q + b + 1) - q0;
  const int tq = kRows / p.n_rep, tok0 = qt * tq;
  if (tok0 >= nq) return -1;
  const int sk = p.seqlens_k != nullptr ? __ldg(p.seqlens_k + b) : nq;
  const int last_tok = min(tok0 + tq, nq) - 1;
  const int kv_end = p.causal ? min(sk, sk - nq + last_tok + 1) : sk;
  return kv_end > 0 ? (kv_end + kBN - 1) / kBN : 0;
}

template <typename T, bool PAGED>
__global__ void __launch_bounds__(kThreads, 1) prefill_tc_kernel(const __grid_constant__ TcKernelArgs args) {
  const PrefillTcParams& p = args.p;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* qs = smem;                        // kGroups Q tiles
  uint8_t* ks = qs + kGroups * kQBytes;      // kNK buffers
  uint8_t* vs = ks + kNK * kKVBytes;         // kNV buffers
  uint64_t* bars = reinterpret_cast<uint64_t*>(vs + kNV * kKVBytes);
  // bars: k_full[kNK], v_full[kNV], k_free[kNK], v_free[kNV], s_full[g], p_full[g], o_done[g]
  constexpr int kBarCount = 2 * (kNK + kNV) + 3 * kGroups;
  static_assert(kBarCount <= 30, "barrier area");
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kBarCount);
  int* s_fail = reinterpret_cast<int*>(tmem_slot + 1);
  // per group and tile parity: j + 1 when tile j of the group needs the lo part of P
  int* s_lo = reinterpret_cast<int*>(bars + 16);
  static_assert(kBarCount + 1 <= 16, "s_lo follows the barriers, TMEM slot and failure flag");
  int* s_pages = reinterpret_cast<int*>(bars + 32);
  float* s_mx = reinterpret_cast<float*>(s_pages + kMaxPagesSmem);  // [group][2 buffers][kSplit][kBM]
  float* s_l = s_mx + kGroups * 2 * kSplit * kBM;                      // [group][kSplit][kBM]

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // ---- work item of this CTA: longest first ----
  // CTA c takes (q-tile item of rank c / Hkv, kv head c % Hkv), items ranked by
  // their number of K/V tiles, descending (ties: lower index first), so the
  // long causal tiles of long requests start in the first wave instead of
  // forming the tail.  Beyond kMaxRanked items the natural order is kept.
  const int n_items = p.B * p.tiles_per_req;
  const int hkv = static_cast<int>(blockIdx.x % p.Hkv);
  int item = static_cast<int>(blockIdx.x / p.Hkv);
  if (n_items <= kMaxRanked) {
    int* s_work = reinterpret_cast<int*>(bars + 32);  // the block-table staging area, not yet in use
    __shared__ int s_item;
    for (int i = tid; i < n_items; i += kThreads) s_work[i] = item_tiles(p, i);
    __syncthreads();
    for (int i = tid; i < n_items; i += kThreads) {
      const int wi = s_work[i];
      int rank = 0;
      for (int j = 0; j < n_items; ++j) {
        const int wj = s_work[j];
        rank += (wj > wi) || (wj == wi && j < i);
      }
      if (rank == item) s_item = i;
    }
    __syncthreads();
    item = s_item;
  }
  const int b = item / p.tiles_per_req;
  const int qt = item % p.tiles_per_req;
  const int q0 = p.cu_q[b];
  const int nq = p.cu_q[b + 1] - q0;
  const int TQg = kBM / p.n_rep;  // query tokens per group
  const int tok0 = qt * kGroups * TQg;
  if (tok0 >= nq) return;  // uniform across the CTA: before any barrier or TMEM use
  const int sk = PAGED ? p.seqlens_k[b] : nq;
  const T* qg = reinterpret_cast<const T*>(p.q);
  const T* kg = reinterpret_cast<const T*>(p.k);
  const T* vg = reinterpret_cast<const T*>(p.v);
  auto k_full = [&](int t) { return smem_u32(&bars[t % kNK]); };
  auto v_full = [&](int t) { return smem_u32(&bars[kNK + t % kNV]); };
  auto k_free = [&](int t) { return smem_u32(&bars[kNK + kNV + t % kNK]); };
  auto v_free = [&](int t) { return smem_u32(&bars[2 * kNK + kNV + t % kNV]); };
  auto s_full = [&](int g) { return smem_u32(&bars[2 * (kNK + kNV) + g]); };
  auto p_full = [&](int g) { return smem_u32(&bars[2 * (kNK + kNV) + kGroups + g]); };
  auto o_done = [&](int g) { return smem_u32(&bars[2 * (kNK + kNV) + 2 * kGroups + g]); };

  if (warp == 0) {
    tc::tmem_alloc(smem_u32(tmem_slot), kTmemCols);
    tc::tmem_relinquish();
  }
  if (tid == 0) {
    for (int i = 0; i < kNK; ++i) {
      tc::mbar_init(k_full(i), PAGED ? 1u : 32u);
      tc::mbar_init(k_free(i), 1u);
    }
    for (int i = 0; i < kNV; ++i) {
      tc::mbar_init(v_full(i), PAGED ? 1u : 32u);
      tc::mbar_init(v_free(i), 1u);
    }
    for (int g = 0; g < kGroups; ++g) {
      tc::mbar_init(s_full(g), 1u);
      tc::mbar_init(p_full(g), 32u * kGroupWarps);
      tc::mbar_init(o_done(g), 1u);
    }
    *s_fail = 0;
    for (int i = 0; i < 2 * kGroups; ++i) s_lo[i] = 0;
    tc::fence_mbar_init();
  }

  const int last_tok = min(tok0 + kGroups * TQg, nq) - 1;
  const int kv_end = p.causal ? min(sk, sk - nq + last_tok + 1) : sk;
  const int n_tiles = kv_end > 0 ? (kv_end + kBN - 1) / kBN : 0;
  if constexpr (PAGED) {
    const int np = min((kv_end + kPage - 1) / kPage, kMaxPagesSmem);
    for (int i = tid; i < np; i += kThreads) s_pages[i] = __ldg(p.bt + static_cast<int64_t>(b) * p.bt_sb + i);
  }
  // ---- Q tiles -> shared memory, 128-B swizzled K-major: group g row m = (token
  //      tok0 + g*TQg + m / n_rep, head m % n_rep); [d-block][row][128 B] per group ----
  if (tid < kRows) {
    const int g = tid / kBM, m = tid % kBM;
    const int tq = tok0 + g * TQg + m / p.n_rep, r = m % p.n_rep;
    const uint4* src = reinterpret_cast<const uint4*>(qg + (static_cast<int64_t>(q0 + tq) * p.Hq + hkv * p.n_rep + r) * kD);
    uint8_t* qd = qs + g * kQBytes;
#pragma unroll
    for (int ch = 0; ch < kD / 8; ++ch) {
      const uint4 v = tq < nq ? __ldg(src + ch) : make_uint4(0, 0, 0, 0);
      *reinterpret_cast<uint4*>(qd + (ch >> 3) * (kBM * 128) + sw_off(m, ch & 7)) = v;
    }
    tc::fence_proxy_async_smem();
  }
  tc::tc_fence_before();
  __syncthreads();  // barriers initialised, TMEM address published, block table and Q staged
  tc::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  auto t_s = [&](int g) { return tmem + static_cast<uint32_t>(g * 256); };
  auto t_o = [&](int g) { return tmem + static_cast<uint32_t>(g * 256 + 128); };
  constexpr bool kBf16 = SplitP<T>::value;

  if (warp >= kLoadWarp) {
    // =================== producer warps: loads (warp 16), MMA issue (warp 17) ===================
    // K (which = 0) or V (which = 1) of tile t into its ring buffer
    auto load_kv = [&](int t, int which) {
      uint8_t* base = which == 0 ? ks + (t % kNK) * kKVBytes : vs + (t % kNV) * kKVBytes;
      const uint32_t bar = which == 0 ? k_full(t) : v_full(t);
      if constexpr (PAGED) {
        // lane (pg, db) = (lane >> 1, lane & 1) issues the box of page pg, head_dim half db
        const CUtensorMap* map = which == 0 ? &args.tmap_k : &args.tmap_v;
        const int pg0 = t * (kBN / kPage);
        const int npg = min(kBN / kPage, (kv_end - pg0 * kPage + kPage - 1) / kPage);
        if (lane == 0) mbar_expect_tx(bar, static_cast<uint32_t>(npg * kDB * kPage * 128));
        __syncwarp();
        if (lane < npg * kDB) {
          const int pg = lane >> 1, db = lane & 1;
          const int idx = pg0 + pg;
          const int page = idx < kMaxPagesSmem ? s_pages[idx] : __ldg(p.bt + static_cast<int64_t>(b) * p.bt_sb + idx);
          tma_load_4d(smem_u32(base + db * (kBN * 128) + pg * kPage * 128), map, db * 64, hkv, 0, page, bar);
        }
      } else {
        const T* src0 = which == 0 ? kg : vg;
        for (int ci = lane; ci < kBN * (kD / 8); ci += 32) {
          const int tt = ci / (kD / 8), ch = ci % (kD / 8);
          const int tk = t * kBN + tt;
          const bool ok = tk < kv_end;
          const int64_t off = ok ? (static_cast<int64_t>(q0 + tk) * p.Hkv + hkv) * kD + ch * 8 : 0;
          cp_async16(smem_u32(base + (ch >> 3) * (kBN * 128) + sw_off(tt, ch & 7)),
                     ok ? (const void*)(src0 + off) : (const void*)src0, ok);
        }
        cp_async_arrive(bar);
      }
    };
    const uint32_t id_s = tc::idesc_f16(kBf16, false, false, kBM, kBN);
    const uint32_t id_o = tc::idesc_f16(kBf16, false, true, kBM, kD);
    // Descriptors are built once; per k-step only the start-address field (bits
    // 0-13, address >> 4) advances, which stays inside the field for smem < 256 KB.
    const uint64_t dq0 = tc::smem_desc_sw128(smem_u32(qs), 16, 1024);
    const uint64_t dk0 = tc::smem_desc_sw128(smem_u32(ks), 16, 1024);
    const uint64_t dv0 = tc::smem_desc_sw128(smem_u32(vs), kBN * 128, 1024);
    auto issue_s = [&](int g, int j) {  // S_g(j) = Q_g K(j)^T, both operands in shared memory
      tc::tc_fence_after();
      const uint64_t qb = dq0 + static_cast<uint64_t>((g * kQBytes) >> 4);
      const uint64_t kb = dk0 + static_cast<uint64_t>(((j % kNK) * kKVBytes) >> 4);
#pragma unroll
      for (int kk = 0; kk < kD / 16; ++kk) {
        const uint64_t qoff = static_cast<uint64_t>(((kk >> 2) * (kBM * 128) + (kk & 3) * 32) >> 4);
        const uint64_t kboff = static_cast<uint64_t>(((kk >> 2) * (kBN * 128) + (kk & 3) * 32) >> 4);
        tc::mma_f16(t_s(g), qb + qoff, kb + kboff, id_s, kk > 0 ? 1u : 0u);
      }
      tc::mma_commit(s_full(g));
    };
    auto issue_o = [&](int g, int j) {  // O_g += P_g(j) V(j), P_g from TMEM (bf16: hi part, then lo part if needed)
      tc::tc_fence_after();
      const uint64_t vb = dv0 + static_cast<uint64_t>(((j % kNV) * kKVBytes) >> 4);
      // the softmax warps of group g marked tile j (before their p_full arrival) if it needs lo
      const int parts = (kBf16 && kSplitPBf16 && s_lo[g * 2 + (j & 1)] == j + 1) ? 2 : 1;
      for (int part = 0; part < parts; ++part) {
#pragma unroll
        for (int kk = 0; kk < kBN / 16; ++kk) {
          const uint32_t pa = t_s(g) + (kk >> 1) * 32 + part * 16 + (kk & 1) * 8;
          tc::mma_f16_ts(t_o(g), pa, vb + static_cast<uint64_t>((kk * 16 * 128) >> 4), id_o,
                         (j > 0 || part > 0 || kk > 0) ? 1u : 0u);
        }
      }
      tc::mma_commit(o_done(g));
    };
    bool ok = true;
    if (warp == kLoadWarp) {
      for (int t = 0; t < kNK - 1 && t < n_tiles; ++t) load_kv(t, 0);
      for (int t = 0; t < kNV - 1 && t < n_tiles; ++t) load_kv(t, 1);
      for (int j = 0; ok && j < n_tiles; ++j) {
        if (j + kNK - 1 < n_tiles) {  // K buffer of tile j-1: free once S_B(j-1) completed
          if (j >= 1) ok = tc::mbar_wait(k_free(j - 1), ((j - 1) / kNK) & 1);
          if (!ok) break;
          load_kv(j + kNK - 1, 0);
        }
        if (j + kNV - 1 < n_tiles) {  // V buffer of tile j-1: free once PV_B(j-1) completed
          if (j >= 1) ok = tc::mbar_wait(v_free(j - 1), ((j - 1) / kNV) & 1);
          if (!ok) break;
          load_kv(j + kNV - 1, 1);
        }
        __syncwarp();
      }
    } else {
      // Tensor-pipe order: S_A(0) S_B(0) | PV_A(0) S_A(1) PV_B(0) S_B(1) | PV_A(1) S_A(2) ...
      // S_g(j+1) overwrites P_g(j), so it is issued once PV_g(j) has completed; between
      // P_g(j) and PV_g(j+1) the pipe runs the other group's PV and S (the window in
      // which group g computes its softmax).
      if (n_tiles > 0) {
        ok = tc::mbar_wait(k_full(0), 0);
        if (ok && lane == 0) {
          issue_s(0, 0);
          issue_s(1, 0);
          tc::mma_commit(k_free(0));
        }
        __syncwarp();
      }
#ifdef BPKV_TRACE
      long long _tm = clock64();
#endif
      for (int j = 0; ok && j < n_tiles; ++j) {
        const uint32_t par = j & 1;
        BPKV_MARK_MMA(20);
        ok = tc::mbar_wait(p_full(0), par) && tc::mbar_wait(v_full(j), (j / kNV) & 1);
        if (!ok) break;
        BPKV_MARK_MMA(21);
        if (lane == 0) issue_o(0, j);
        __syncwarp();
        BPKV_MARK_MMA(22);
        if (j + 1 < n_tiles) {
          ok = tc::mbar_wait(k_full(j + 1), ((j + 1) / kNK) & 1) && tc::mbar_wait(o_done(0), par);
          if (!ok) break;
          BPKV_MARK_MMA(23);
          if (lane == 0) issue_s(0, j + 1);
          __syncwarp();
          BPKV_MARK_MMA(24);
        }
        ok = tc::mbar_wait(p_full(1), par);
        if (!ok) break;
        BPKV_MARK_MMA(25);
        if (lane == 0) {
          issue_o(1, j);
          tc::mma_commit(v_free(j));
        }
        __syncwarp();
        BPKV_MARK_MMA(26);
        if (j + 1 < n_tiles) {
          ok = tc::mbar_wait(o_done(1), par);
          if (!ok) break;
          BPKV_MARK_MMA(27);
          if (lane == 0) {
            issue_s(1, j + 1);
            tc::mma_commit(k_free(j + 1));
          }
          __syncwarp();
        }
      }
    }
    if (!ok) *s_fail = 1;
  } else {
    // ============ softmax warps: group g = warp / 8, kSplit threads per accumulator row ============
    // warp w of group g handles rows (w % 4)*32 + lane (TMEM lanes of its sub-partition) and
    // column half h = (w % 8) / 4: S columns [64h, 64h+64) of S_g, O columns [64h, 64h+64) of O_g.
    const int g = warp / kGroupWarps;
    const int half = (warp % kGroupWarps) / 4;
    const int rq = warp % 4;
    const int row = rq * 32 + lane;
    const int tok = tok0 + g * TQg + row / p.n_rep;
    const int lim = p.causal ? (tok < nq ? sk - nq + tok : sk - 1) : sk - 1;
    const uint32_t lane_base = static_cast<uint32_t>(rq * 32) << 16;
    constexpr int kSC = kBN / kSplit, kOC = kD / kSplit;
    static_assert(kSC == 64 && kOC == 64, "two x32 TMEM loads per thread and tile");
    const int sc0 = half * kSC, oc0 = half * kOC;
    const uint32_t ts = t_s(g) + lane_base + sc0, to = t_o(g) + lane_base + oc0;
    const uint32_t bar_id = 2 + g * 4 + rq;  // the kSplit warps sharing these rows
    float* mxg = s_mx + g * 2 * kSplit * kBM;
    float m_ref = -INFINITY, l_run = 0.f;
    // A failed (timed-out) wait only sets `failed`: the loop keeps its shape, so
    // every softmax warp still reaches every named barrier, and later waits are
    // skipped; the rows are then written as NaN.
    bool failed = false;
    auto wait = [&](uint32_t bar, uint32_t parity) {
      if (failed) return;
      const bool r = tc::mbar_wait(bar, parity);
      if (!__all_sync(0xffffffffu, r)) failed = true;
    };
#ifdef BPKV_TRACE
    long long _tl = clock64();
    const long long _tstart = _tl;
#endif
    for (int it = 0; it < n_tiles; ++it) {
      // S_g(it) complete; its commit also covers PV_g(it-1), so O_g and the P_g area are free
      wait(s_full(g), it & 1);
      BPKV_MARK(0);
      tc::tc_fence_after();
      const int tbase = it * kBN + sc0;
      const bool crosses = tbase + kSC - 1 > lim;  // only tiles that cross this row's causal limit need the mask
      // pass 1: row maximum over this thread's 64 columns; columns [32, 64) stay in registers for
      // pass 2, which reads only [0, 32) again
      float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};  // four independent max chains
      float s1[32];
      {
        float s0[32];
        tc::tmem_ld32x2(ts, ts + 32, s0, s1);
        if (crosses) {
#pragma unroll
          for (int c = 0; c < 32; ++c) {
            s0[c] = (tbase + c <= lim) ? s0[c] : -INFINITY;
            s1[c] = (tbase + 32 + c <= lim) ? s1[c] : -INFINITY;
          }
        }
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          mx4[c & 3] = fmaxf(mx4[c & 3], s0[c]);
          mx4[c & 3] = fmaxf(mx4[c & 3], s1[c]);
        }
      }
      BPKV_MARK(1);
      const float mxh = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3]));
      BPKV_MARK(2);
      // exchange the half-row maxima with the partner warp (double-buffered)
      mxg[((it & 1) * kSplit + half) * kBM + row] = mxh;
      // bf16: can this tile's P go to the P.V MMA as one bf16 part?  Yes when, in every row of
      // the group, its largest weight is at most 2^-kLoLog2 (2^-8) of the row sum so far
      // (scale-free: both in units of 2^m_ref; this thread's half-row sum is a lower bound of
      // the row sum): each weight then keeps a bf16 rounding error <= 2^-9 * 2^-8 of the final
      // sum, and the random sum of those errors stays far inside the 2e-3 bar.  Measured at
      // config-5 shapes: 2.4e-4 max-abs against fp64 as with the split everywhere (7.7e-4 with
      // no split); 2^-6 ran 6% faster but was less accurate than flash-attn's bf16 P on one
      // chunk.  Otherwise (early tiles, few or dominant keys) the hi/lo split keeps ~16 bits.
      // One group-wide AND at the max-exchange barrier.
      bool need_lo = kBf16 && kSplitPBf16;
      if constexpr (kBf16 && kSplitPBf16) {
        const float mxh_s = mxh * p.scale_log2;
        const uint32_t small =
            (mxh_s == -INFINITY) || (m_ref != -INFINITY && l_run > 0.f && mxh_s - m_ref <= __log2f(l_run) - kLoLog2);
        uint32_t all_small;
        asm volatile(
            "{\n .reg .pred pc, pr;\n setp.ne.u32 pc, %1, 0;\n bar.red.and.pred pr, %2, %3, pc;\n"
            " selp.u32 %0, 1, 0, pr;\n}\n"
            : "=r"(all_small)
            : "r"(small), "r"(10 + g), "n"(32 * kGroupWarps)
            : "memory");
        need_lo = all_small == 0;
        if (need_lo && (warp % kGroupWarps) == 0 && lane == 0) s_lo[g * 2 + (it & 1)] = it + 1;
      } else {
        asm volatile("bar.sync %0, %1;\n" ::"r"(bar_id), "n"(32 * kSplit) : "memory");
      }
      float mxr = mxg[((it & 1) * kSplit) * kBM + row];
#pragma unroll
      for (int h = 1; h < kSplit; ++h) mxr = fmaxf(mxr, mxg[((it & 1) * kSplit + h) * kBM + row]);
      const float mx = mxr * p.scale_log2;
      BPKV_MARK(3);
      // lazy reference max: move it (rescale O, l) only when the row max grew by > threshold
      const bool need = mx > m_ref + kRescaleThreshold;
      float alpha = 1.f;
      if (need) {
        alpha = fast_exp2(m_ref - mx);  // 0 when m_ref = -inf
        m_ref = mx;
        l_run *= alpha;
      }
      BPKV_MARK(4);
      const float m_use = m_ref == -INFINITY ? 0.f : m_ref;
      const uint64_t sc2 = pk2(p.scale_log2, p.scale_log2), nm2 = pk2(-m_use, -m_use);
      uint64_t sum2[2] = {0ull, 0ull};  // two independent packed sum chains (0ull = +0.0f pair)
      // pass 2, chunk by chunk: S columns [c0, c0+32) -> P hi / lo in the same 32 columns; chunk
      // [32, 64) first, from the registers of pass 1 (its P stores never touch columns [0, 32))
      auto emit = [&](int c0, float* s) {
        uint32_t hi[16], lo[16];
#pragma unroll
        for (int c = 0; c < 32; c += 2) {
          const uint64_t x2 = fma2(pk2(s[c], s[c + 1]), sc2, nm2);
          uint64_t e2;
          if ((c >> 1) % kEmuStride == kEmuStride - 1) {
            e2 = exp2_poly2(x2);
          } else {
            float xa, xb;
            up2(x2, xa, xb);
            e2 = pk2(fast_exp2(xa), fast_exp2(xb));
          }
          sum2[(c >> 1) & 1] = add2(sum2[(c >> 1) & 1], e2);
          float ea, eb;
          up2(e2, ea, eb);
          if (kBf16 && kSplitPBf16 && need_lo) {
            // hi = bf16(e), lo = bf16(e - hi); bf16 -> fp32 is a 16-bit shift
            const uint32_t h = pack2<T>(ea, eb);
            const uint64_t l2 = sub2(e2, pk2(__uint_as_float(h << 16), __uint_as_float(h & 0xffff0000u)));
            float la, lb;
            up2(l2, la, lb);
            hi[c >> 1] = h;
            lo[c >> 1] = pack2<T>(la, lb);
          } else {
            hi[c >> 1] = pack2<T>(ea, eb);
            lo[c >> 1] = 0u;
          }
        }
        // P_g(it) over this chunk of S_g: token pair per 32-bit column, hi parts then lo parts
        tc::tmem_st16_nowait(ts + c0, hi);
        if (kBf16 && kSplitPBf16 && need_lo) tc::tmem_st16_nowait(ts + c0 + 16, lo);
      };
      emit(32, s1);
      {
        float s0[32];
        tc::tmem_ld32(ts, s0);
        if (crosses) {
#pragma unroll
          for (int c = 0; c < 32; ++c) s0[c] = (tbase + c <= lim) ? s0[c] : -INFINITY;
        }
        emit(0, s0);
      }
      // O rescale (rare: the reference max moved) after P, so S and O are not held together
      if (it > 0 && __any_sync(0xffffffffu, need)) {
#pragma unroll
        for (int c0 = 0; c0 < kOC; c0 += 32) {
          float o[32];
          tc::tmem_ld32(to + c0, o);
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] *= alpha;
          tmem_st32(to + c0, o);
        }
      }
      tc::tmem_st_wait();  // all P (and O) stores of this tile complete before the arrival below
      BPKV_MARK(5);
      {
        float sa, sb;
        up2(add2(sum2[0], sum2[1]), sa, sb);
        l_run += sa + sb;
      }
      bool zeroed = false;
      if (g == 0 && it == n_tiles - 1 && kv_end < (it + 1) * kBN) {
        // rows of the last page past kv_end hold whatever the pool page holds (P is
        // 0 there, but 0 * NaN is not): zero them in the V tile once it has landed;
        // PV_A(it) and PV_B(it) both come after this group's arrival on p_full
        wait(v_full(it), (it / kNV) & 1);
        uint8_t* vb = vs + (it % kNV) * kKVBytes;
        const int first = kv_end - it * kBN;
        for (int e = tid; e < (kBN - first) * kDB * 8; e += 32 * kGroupWarps) {
          const int tt = first + e / (kDB * 8), rem = e % (kDB * 8);
          *reinterpret_cast<uint4*>(vb + (rem >> 3) * (kBN * 128) + tt * 128 + (rem & 7) * 16) =
              make_uint4(0, 0, 0, 0);
        }
        zeroed = true;
      }
      if (zeroed) tc::fence_proxy_async_smem();  // zeroed V rows -> visible to the tensor core
      tc::tc_fence_before();                     // P stores in TMEM -> ordered before the MMA warp's issue
      asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(p_full(g)) : "memory");
      BPKV_MARK(6);
    }
    if (n_tiles > 0) wait(o_done(g), (n_tiles - 1) & 1);
#ifdef BPKV_TRACE
    if (BPKV_TRACING && tid == 0) {
      atomicAdd(&g_prefill_trace[11], static_cast<unsigned long long>(clock64() - _tstart));
      atomicAdd(&g_prefill_trace[10], static_cast<unsigned long long>(n_tiles));
    }
#endif
    if (failed) *s_fail = 1;
    const bool ok = !failed;
    // ---- epilogue: row sum of both halves, O / l from TMEM ----
    float* lg = s_l + g * kSplit * kBM;
    lg[half * kBM + row] = l_run;
    asm volatile("bar.sync %0, %1;\n" ::"r"(bar_id), "n"(32 * kSplit) : "memory");
    float l_row = 0.f;
#pragma unroll
    for (int h = 0; h < kSplit; ++h) l_row += lg[h * kBM + row];
    const bool all_ok = __all_sync(0xffffffffu, ok);  // before any divergent branch
    const float inv = l_row > 0.f ? 1.f / l_row : 0.f;
    const float nan = __int_as_float(0x7fc00000);
    T* dst = reinterpret_cast<T*>(p.out) +
             (static_cast<int64_t>(q0 + tok) * p.Hq + hkv * p.n_rep + row % p.n_rep) * kD + oc0;
    if (all_ok && n_tiles > 0) tc::tc_fence_after();
#pragma unroll
    for (int c0 = 0; c0 < kOC; c0 += 32) {
      float acc[32];
      if (all_ok && n_tiles > 0) {
        tc::tmem_ld32(to + c0, acc);
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) acc[i] = 0.f;
      }
      if (tok < nq) {
#pragma unroll
        for (int c = 0; c < 32; c += 8) {
          float v[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) v[i] = all_ok ? acc[c + i] * inv : nan;
          *reinterpret_cast<uint4*>(dst + c0 + c) =
              make_uint4(pack2<T>(v[0], v[1]), pack2<T>(v[2], v[3]), pack2<T>(v[4], v[5]), pack2<T>(v[6], v[7]));
        }
      }
    }
  }
  cp_async_wait<0>();
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, kTmemCols);
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

// 4-D view of one pool layer: (head_dim, kv_head, token-in-page, page); one
// box = 64 elements of head_dim x 1 head x 16 tokens of one page, 128-B swizzle.
bool make_page_map(CUtensorMap* map, const void* base, int Hkv, int64_t page_stride, bool bf16) {
  EncodeTiledFn enc = encode_fn();
  if (enc == nullptr) return false;
  const cuuint64_t dims[4] = {static_cast<cuuint64_t>(kD), static_cast<cuuint64_t>(Hkv), 16, 1u << 24};
  const cuuint64_t strides[3] = {static_cast<cuuint64_t>(kD) * 2, static_cast<cuuint64_t>(Hkv) * kD * 2,
                                 static_cast<cuuint64_t>(page_stride) * 2};
  const cuuint32_t box[4] = {64, 1, 16, 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  return enc(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<void*>(base),
             dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

// Launches the tcgen05 kernel; returns BPKV_ERR_UNSUPPORTED when the shape is
// not one it handles (head_dim 128, bf16/fp16, n_rep dividing 128).
int prefill_tc_launch(PrefillTcParams& p, int head_dim, int dtype, int max_seqlen_q, bool paged, cudaStream_t st) {
  if (head_dim != kD || (dtype != BPKV_BF16 && dtype != BPKV_F16) || kBM % p.n_rep != 0) return BPKV_ERR_UNSUPPORTED;
  if (paged && (p.page_stride * 2) % 16 != 0) return BPKV_ERR_UNSUPPORTED;
  const int TQ = kRows / p.n_rep;  // query tokens per CTA
  p.tiles_per_req = (max_seqlen_q + TQ - 1) / TQ;
  if (p.tiles_per_req == 0 || p.B == 0) return BPKV_OK;
  TcKernelArgs args;
  memset(&args, 0, sizeof(args));
  args.p = p;
  if (paged) {
    if (!make_page_map(&args.tmap_k, p.k, p.Hkv, p.page_stride, dtype == BPKV_BF16) ||
        !make_page_map(&args.tmap_v, p.v, p.Hkv, p.page_stride, dtype == BPKV_BF16)) {
      set_error("prefill_tc_launch:tensor_map_encode_failed");
      return BPKV_ERR_CUDA;
    }
  }
  dim3 grid(p.B * p.tiles_per_req * p.Hkv);
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
    kern<<<grid, kThreads, kSmemBytes, st>>>(args);                                                             \
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

#ifdef BPKV_TRACE
extern "C" BPKV_API int bpkv_debug_prefill_trace(unsigned long long* out, int n, int reset) {
  if (n > 32) n = 32;
  if (cudaMemcpyFromSymbol(out, bpkv::g_prefill_trace, sizeof(unsigned long long) * n) != cudaSuccess) return 3;
  if (reset) {
    unsigned long long z[32] = {0};
    cudaMemcpyToSymbol(bpkv::g_prefill_trace, z, sizeof(z));
  }
  return 0;
}
#endif
