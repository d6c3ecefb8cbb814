// Split-KV merge over NVLink peer memory of partials that the caller already
// holds (one (out, lse) per rank), replacing the NCCL all-gather of packed
// partials + the merge kernel of the long-sequence decode (one sequence whose
// pages are split across GPUs).  The exchange buffer and its word format are
// described in peer_words.cuh; the decode path that produces its own fp32
// partials and merges them in the same kernel is bpkv_split_kv_decode_p2p
// (page16_decode.cu).
//
// peer_exchange_kernel<TP, TO>, one launch per call, a programmatic dependent
// launch of whatever produced the partial (it waits for that grid first):
//   CTA c owns rows [8c, 8c+8).  It stores those rows of this rank's partial
//   (TP out converted to fp32, fp32 lse) into every peer's buffer with plain
//   16-byte stores through the IPC mapping (NVLink), then merges them, one
//   warp per row: the lse words of every other rank first (bounded spin on
//   their call number), M = max lse, W = sum exp(lse - M), then out = sum
//   exp(lse - M) o / W (written as TO) and lse_out = M + log W, each other
//   rank's words read with the same bounded spin.  The own partial is read in
//   place.  The last CTA to finish advances the call number.
// A wait that runs out sets *status = 1 and writes NaN rows; the context stays
// usable.  No multicast, no TMA: plain loads and stores.
#include "peer_words.cuh"

namespace bpkv {
namespace {

using peer::kMaxRanks;
constexpr int kRowsPerCta = 8;  // one merging warp per row
constexpr int kThreads = kRowsPerCta * 32;

struct PeerArgs {
  uint4* bufs[kMaxRanks];  // every rank's exchange buffer as mapped in this process (own included)
  const void* part_out;    // [rows][D] this rank's partial output (TP)
  const float* part_lse;   // [rows] natural-log sum-exp of this rank's partial
  void* out;               // [rows][D] merged output (TO)
  float* lse_out;          // [rows] or null
  int* status;             // 0 ok, 1 a wait ran out
  int rank, world, rows, D;
  uint32_t max_polls;
};

template <typename TP, typename TO>
__global__ void __launch_bounds__(kThreads) peer_exchange_kernel(const __grid_constant__ PeerArgs a) {
  pdl_wait();  // the partial comes from the preceding grid
  uint4* own = a.bufs[a.rank];
  const uint32_t epoch = *peer::epoch_ptr(own, a.world, a.rows, a.D) + 1u;  // this call
  const int par = static_cast<int>(epoch & 1u);
  const int W = static_cast<int>(peer::row_words(a.D)), H = a.D / 2;
  const int r0 = blockIdx.x * kRowsPerCta, r1 = min(a.rows, r0 + kRowsPerCta);
  const TP* src = reinterpret_cast<const TP*>(a.part_out);
  // ---- 1. send this CTA's rows to every peer ----
  const int n_words = (r1 - r0) * W;
  for (int e = threadIdx.x; e < (a.world - 1) * n_words; e += blockDim.x) {
    const int i = e / n_words, rem = e % n_words;
    const int p = (a.rank + 1 + i) % a.world;
    const int r = r0 + rem / W, j = rem % W;
    float x0, x1;
    if (j < H) {
      x0 = Elem<TP>::to_f(src[static_cast<int64_t>(r) * a.D + 2 * j]);
      x1 = Elem<TP>::to_f(src[static_cast<int64_t>(r) * a.D + 2 * j + 1]);
    } else {
      x0 = a.part_lse[r];
      x1 = 0.f;
    }
    peer::st_word(peer::row_ptr(a.bufs[p], a.world, a.rows, a.D, par, a.rank, r) + j, x0, x1, epoch);
  }
  // ---- 2. merge, one warp per row ----
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = r0 + warp;
  if (r < r1) {
    TO* out = reinterpret_cast<TO*>(a.out) + static_cast<int64_t>(r) * a.D;
    const TP* mine = src + static_cast<int64_t>(r) * a.D;
    const float nan = __int_as_float(0x7fc00000);
    const uint64_t t0 = peer::now_ns();
    uint32_t polls = 0;
    bool ok = true;
    // lane q < world holds rank q's lse
    float lq = -INFINITY;
    if (lane < a.world) {
      if (lane == a.rank) {
        lq = a.part_lse[r];
      } else {
        float unused;
        ok = peer::wait_word(peer::row_ptr(own, a.world, a.rows, a.D, par, lane, r) + H, epoch, polls,
                             a.max_polls, t0, lq, unused);
      }
    }
    float wts[kMaxRanks];
    float M = -INFINITY;
    bool all_ok = __all_sync(0xffffffffu, ok);
    if (all_ok) {
#pragma unroll
      for (int q = 0; q < kMaxRanks; ++q) M = fmaxf(M, __shfl_sync(0xffffffffu, lq, q));
    }
    float Wsum = 0.f;
#pragma unroll
    for (int q = 0; q < kMaxRanks; ++q) {
      const float l = __shfl_sync(0xffffffffu, lq, q);
      wts[q] = (q < a.world && M != -INFINITY) ? expf(l - M) : 0.f;
      Wsum += wts[q];
    }
    if (all_ok && M != -INFINITY) {
      const float invW = 1.f / Wsum;
      for (int j = lane; j < H; j += 32) {
        float acc0 = 0.f, acc1 = 0.f;
#pragma unroll
        for (int q = 0; q < kMaxRanks; ++q) {
          if (q >= a.world || !(wts[q] > 0.f)) continue;
          float v0, v1;
          if (q == a.rank) {
            v0 = Elem<TP>::to_f(mine[2 * j]);
            v1 = Elem<TP>::to_f(mine[2 * j + 1]);
          } else if (!peer::wait_word(peer::row_ptr(own, a.world, a.rows, a.D, par, q, r) + j, epoch, polls,
                                      a.max_polls, t0, v0, v1)) {
            ok = false;
            v0 = v1 = 0.f;
          }
          acc0 += wts[q] * v0;
          acc1 += wts[q] * v1;
        }
        out[2 * j] = Elem<TO>::from_f(acc0 * invW);
        out[2 * j + 1] = Elem<TO>::from_f(acc1 * invW);
      }
      all_ok = __all_sync(0xffffffffu, ok);
      if (all_ok && a.lse_out != nullptr && lane == 0) a.lse_out[r] = M + logf(Wsum);
    } else if (all_ok) {  // no rank had keys for this row (the reference's 0/0)
      for (int d = lane; d < a.D; d += 32) out[d] = Elem<TO>::from_f(nan);
      if (a.lse_out != nullptr && lane == 0) a.lse_out[r] = -INFINITY;
    }
    if (!all_ok) {
      for (int d = lane; d < a.D; d += 32) out[d] = Elem<TO>::from_f(nan);
      if (a.lse_out != nullptr && lane == 0) a.lse_out[r] = nan;
      if (lane == 0) atomicExch(a.status, 1);
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) peer::finish_call(own, a.world, a.rows, a.D, epoch);
}

template <typename TP>
cudaError_t launch_exchange_tp(int out_dtype, dim3 grid, cudaStream_t st, const PeerArgs& a) {
  if (out_dtype == BPKV_BF16) return launch_pdl(peer_exchange_kernel<TP, __nv_bfloat16>, grid, dim3(kThreads), 0, st, a);
  if (out_dtype == BPKV_F16) return launch_pdl(peer_exchange_kernel<TP, __half>, grid, dim3(kThreads), 0, st, a);
  return launch_pdl(peer_exchange_kernel<TP, float>, grid, dim3(kThreads), 0, st, a);
}

cudaError_t launch_exchange(int dtype, int out_dtype, dim3 grid, cudaStream_t st, const PeerArgs& a) {
  if (dtype == BPKV_BF16) return launch_exchange_tp<__nv_bfloat16>(out_dtype, grid, st, a);
  if (dtype == BPKV_F16) return launch_exchange_tp<__half>(out_dtype, grid, st, a);
  return launch_exchange_tp<float>(out_dtype, grid, st, a);
}

}  // namespace
}  // namespace bpkv

using namespace bpkv;

extern "C" BPKV_API size_t bpkv_peer_exchange_bytes(int world, int rows, int head_dim) {
  if (world <= 0 || world > kMaxRanks || rows <= 0 || head_dim <= 0) return 0;
  return peer::exchange_bytes(world, rows, head_dim);
}

extern "C" BPKV_API int bpkv_peer_buffer_alloc(size_t bytes, void** ptr, void* ipc_handle) {
  clear_error();
  BPKV_CHECK_ARG(bytes > 0 && ptr != nullptr && ipc_handle != nullptr, "peer_exchange_shape:alloc_args");
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e == cudaSuccess) e = cudaMemset(p, 0, bytes);  // flags and counts start at 0
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    if (p != nullptr) cudaFree(p);
    set_error("peer_exchange_alloc:%s", cudaGetErrorString(e));
    return BPKV_ERR_CUDA;
  }
  memcpy(ipc_handle, &h, sizeof(h));
  *ptr = p;
  return BPKV_OK;
}

extern "C" BPKV_API int bpkv_peer_buffer_open(const void* ipc_handle, void** ptr) {
  clear_error();
  BPKV_CHECK_ARG(ipc_handle != nullptr && ptr != nullptr, "peer_exchange_shape:open_args");
  cudaIpcMemHandle_t h;
  memcpy(&h, ipc_handle, sizeof(h));
  const cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) {
    set_error("peer_exchange_open:%s", cudaGetErrorString(e));
    return BPKV_ERR_CUDA;
  }
  return BPKV_OK;
}

extern "C" BPKV_API int bpkv_peer_buffer_close(void* ptr) {
  clear_error();
  const cudaError_t e = cudaIpcCloseMemHandle(ptr);
  if (e != cudaSuccess) {
    set_error("peer_exchange_close:%s", cudaGetErrorString(e));
    return BPKV_ERR_CUDA;
  }
  return BPKV_OK;
}

extern "C" BPKV_API int bpkv_peer_buffer_free(void* ptr) {
  clear_error();
  const cudaError_t e = cudaFree(ptr);
  if (e != cudaSuccess) {
    set_error("peer_exchange_free:%s", cudaGetErrorString(e));
    return BPKV_ERR_CUDA;
  }
  return BPKV_OK;
}

extern "C" BPKV_API int bpkv_split_kv_merge_p2p(const void* part_out, const float* part_lse, void* const* peer_bufs,
                                                int rank, int world, int rows, int head_dim, uint32_t max_polls,
                                                void* out, float* lse_out, int* status, int dtype, int out_dtype,
                                                void* stream) {
  clear_error();
  BPKV_CHECK_ARG(world >= 1 && world <= kMaxRanks && rank >= 0 && rank < world, "peer_exchange_shape:rank_%d_of_%d",
                 rank, world);
  BPKV_CHECK_ARG(rows > 0 && head_dim > 0 && head_dim % 4 == 0, "peer_exchange_shape:rows_%d_head_dim_%d", rows,
                 head_dim);
  BPKV_CHECK_ARG(part_out && part_lse && peer_bufs && out && status, "peer_exchange_shape:null_pointer");
  BPKV_CHECK_ARG(dtype == BPKV_BF16 || dtype == BPKV_F16 || dtype == BPKV_F32, "peer_exchange_shape:dtype");
  BPKV_CHECK_ARG(out_dtype == BPKV_BF16 || out_dtype == BPKV_F16 || out_dtype == BPKV_F32,
                 "peer_exchange_shape:out_dtype");
  PeerArgs a;
  memset(&a, 0, sizeof(a));
  for (int r = 0; r < world; ++r) {
    BPKV_CHECK_ARG(peer_bufs[r] != nullptr && aligned16(peer_bufs[r]), "peer_exchange_shape:buffer_%d", r);
    a.bufs[r] = static_cast<uint4*>(peer_bufs[r]);
  }
  a.part_out = part_out;
  a.part_lse = part_lse;
  a.out = out;
  a.lse_out = lse_out;
  a.status = status;
  a.rank = rank;
  a.world = world;
  a.rows = rows;
  a.D = head_dim;
  a.max_polls = max_polls;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const dim3 grid((rows + kRowsPerCta - 1) / kRowsPerCta);
  const cudaError_t le = launch_exchange(dtype, out_dtype, grid, st, a);
  if (le != cudaSuccess) {
    set_error("split_kv_merge_p2p_launch:%s", cudaGetErrorString(le));
    return BPKV_ERR_CUDA;
  }
  BPKV_RETURN_LAUNCH("split_kv_merge_p2p_launch");
}
