// Split-KV merge over NVLink peer memory, replacing the NCCL all-gather of
// packed (out, lse) partials + the merge kernel of the long-sequence decode
// (one sequence whose pages are split across GPUs).
//
// Every rank owns one exchange buffer (cudaMalloc'd by this library, exported
// to the other processes by CUDA IPC and mapped there once):
//   float  data[2][world][rows][D + 4]     (out row, lse at column D; 16-B rows)
//   uint32 flag[2][kMaxRanks]              (flag[par][r] = epoch: rank r's data landed)
//   uint32 count[2][kMaxRanks]             (local: finished chunks per peer)
//   uint32 epoch, merged                   (local: calls completed, merge CTAs done)
// Call number e (kept in device memory, so the kernel can be captured in a CUDA
// graph and replayed) uses parity e & 1: a peer may already write call
// e+1 while this rank still merges e; e+2 cannot start before this rank has
// finished e (its send of e+1 comes after).
//
// peer_exchange_kernel<T>, one launch per call:
//   1. CTA u = (peer index i, chunk c) stores chunk c of this rank's partial
//      (T out, fp32 lse) into peer (rank + 1 + i) % world's buffer with plain
//      stores through the IPC mapping (NVLink), fences at system scope, and
//      the last chunk for that peer raises flag[par][rank] = e there with a
//      release store.  The rank's own partial is not copied: the merge reads
//      it in place.
//   2. every CTA waits (bounded spin on acquire loads) until the flags of all
//      other ranks for call e are up in the own buffer.  Those flags are set
//      by the kernels of the other GPUs only, never by a CTA of this grid.
//   3. the CTAs merge rows r = blockIdx.x*8 + warp, stride gridDim.x*8: M =
//      max lse, W = sum exp(lse - M), out = sum exp(lse - M) o / W, lse_out =
//      M + log W; the last CTA to finish advances the call number.
// A wait that runs out sets *status = 1 and writes NaN rows; the context stays
// usable.  No multicast, no TMA: plain loads and stores.
#include "common.cuh"

namespace bpkv {
namespace {

constexpr int kMaxRanks = 8;
constexpr int kSendThreads = 256;

struct PeerArgs {
  float* bufs[kMaxRanks];  // every rank's exchange buffer as mapped in this process (own included)
  const void* part_out;    // [rows][D] this rank's partial output (T)
  const float* part_lse;   // [rows] natural-log sum-exp of this rank's partial
  void* out;               // [rows][D] merged output (T)
  float* lse_out;          // [rows] or null
  int* status;             // 0 ok, 1 a wait ran out
  int rank, world, rows, D, chunks, rows_per_chunk;
  uint32_t max_polls;
};

__host__ __device__ inline int64_t row_floats(int D) { return D + 4; }
__host__ __device__ inline int64_t data_floats(int world, int rows, int D) {
  return 2LL * world * rows * row_floats(D);
}
__device__ inline uint32_t* flag_ptr(float* buf, const PeerArgs& a, int par, int r) {
  return reinterpret_cast<uint32_t*>(buf + data_floats(a.world, a.rows, a.D)) + par * kMaxRanks + r;
}
__device__ inline uint32_t* count_ptr(float* buf, const PeerArgs& a, int par, int p) {
  return reinterpret_cast<uint32_t*>(buf + data_floats(a.world, a.rows, a.D)) + 2 * kMaxRanks + par * kMaxRanks + p;
}
__device__ inline uint32_t* epoch_ptr(float* buf, const PeerArgs& a) {
  return reinterpret_cast<uint32_t*>(buf + data_floats(a.world, a.rows, a.D)) + 4 * kMaxRanks;
}

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;\n" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// One merged row, one warp.  Rank q's partial comes from the own buffer, the
// own rank's from part_out / part_lse in place.
template <typename T>
__device__ void merge_row(const PeerArgs& a, const float* own, int par, int r, bool failed, int lane) {
  T* out = reinterpret_cast<T*>(a.out) + static_cast<int64_t>(r) * a.D;
  const float nan = __int_as_float(0x7fc00000);
  if (failed) {
    for (int d = lane; d < a.D; d += 32) out[d] = Elem<T>::from_f(nan);
    if (a.lse_out != nullptr && lane == 0) a.lse_out[r] = nan;
    return;
  }
  const float* base = own + (static_cast<int64_t>(par) * a.world * a.rows + r) * row_floats(a.D);
  const int64_t slot = static_cast<int64_t>(a.rows) * row_floats(a.D);
  const T* mine = reinterpret_cast<const T*>(a.part_out) + static_cast<int64_t>(r) * a.D;
  float lse[kMaxRanks];
  float M = -INFINITY;
#pragma unroll
  for (int q = 0; q < kMaxRanks; ++q) {
    lse[q] = q >= a.world ? -INFINITY : (q == a.rank ? a.part_lse[r] : base[q * slot + a.D]);
    M = fmaxf(M, lse[q]);
  }
  if (M == -INFINITY) {  // no rank had keys for this row (the reference's 0/0)
    for (int d = lane; d < a.D; d += 32) out[d] = Elem<T>::from_f(nan);
    if (a.lse_out != nullptr && lane == 0) a.lse_out[r] = -INFINITY;
    return;
  }
  float w[kMaxRanks];
  float W = 0.f;
#pragma unroll
  for (int q = 0; q < kMaxRanks; ++q) {
    w[q] = q < a.world ? expf(lse[q] - M) : 0.f;
    W += w[q];
  }
  const float invW = 1.f / W;
  for (int d = lane; d < a.D; d += 32) {
    float acc = 0.f;
#pragma unroll
    for (int q = 0; q < kMaxRanks; ++q) {
      if (q >= a.world || !(w[q] > 0.f)) continue;
      acc += w[q] * (q == a.rank ? Elem<T>::to_f(mine[d]) : base[q * slot + d]);
    }
    out[d] = Elem<T>::from_f(acc * invW);
  }
  if (a.lse_out != nullptr && lane == 0) a.lse_out[r] = M + logf(W);
}

template <typename T>
__global__ void __launch_bounds__(kSendThreads) peer_exchange_kernel(const __grid_constant__ PeerArgs a) {
  __shared__ int s_failed;
  float* own = a.bufs[a.rank];
  const uint32_t epoch = *epoch_ptr(own, a) + 1u;  // this call; stored back by the last CTA below
  const int par = static_cast<int>(epoch & 1u);
  const int n_send = (a.world - 1) * a.chunks;
  // ---- 1. send ----
  if (static_cast<int>(blockIdx.x) < n_send) {
    const int i = blockIdx.x / a.chunks, c = blockIdx.x % a.chunks;
    const int p = (a.rank + 1 + i) % a.world;
    float* dst = a.bufs[p] + ((static_cast<int64_t>(par) * a.world + a.rank) * a.rows) * row_floats(a.D);
    const T* src = reinterpret_cast<const T*>(a.part_out);
    const int r0 = c * a.rows_per_chunk, r1 = min(a.rows, r0 + a.rows_per_chunk);
    const int q4 = a.D / 4;  // float4 per row (D % 4 == 0)
    for (int e = threadIdx.x; e < (r1 - r0) * (q4 + 1); e += blockDim.x) {
      const int r = r0 + e / (q4 + 1), j = e % (q4 + 1);
      float* drow = dst + static_cast<int64_t>(r) * row_floats(a.D);
      if (j < q4) {
        const T* sp = src + static_cast<int64_t>(r) * a.D + 4 * j;
        *reinterpret_cast<float4*>(drow + 4 * j) =
            make_float4(Elem<T>::to_f(sp[0]), Elem<T>::to_f(sp[1]), Elem<T>::to_f(sp[2]), Elem<T>::to_f(sp[3]));
      } else {
        drow[a.D] = a.part_lse[r];
      }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      __threadfence_system();  // this chunk's stores before the count below
      uint32_t* cnt = count_ptr(own, a, par, p);
      if (atomicAdd(cnt, 1u) == static_cast<uint32_t>(a.chunks - 1)) {
        *cnt = 0u;               // ready for call e + 2 (same parity)
        __threadfence_system();  // every chunk's stores (seen through the count) before the flag
        st_release_sys(flag_ptr(a.bufs[p], a, par, a.rank), epoch);
      }
    }
  }
  // ---- 2. wait for the other ranks' partials of this call ----
  if (threadIdx.x == 0) {
    int failed = 0;
    for (int q = 0; q < a.world && !failed; ++q) {
      if (q == a.rank) continue;
      const uint32_t* f = flag_ptr(own, a, par, q);
      uint32_t polls = 0;
      uint64_t t0;
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
      while (static_cast<int32_t>(ld_acquire_sys(f) - epoch) < 0) {
        uint64_t t;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
        if (++polls > a.max_polls || t - t0 > 4000000000ull) {  // poll count or 4 s, whichever first
          failed = 1;
          break;
        }
      }
    }
    s_failed = failed;
    if (failed) atomicExch(a.status, 1);
  }
  __syncthreads();
  // ---- 3. merge ----
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  for (int r = blockIdx.x * nw + warp; r < a.rows; r += gridDim.x * nw) merge_row<T>(a, own, par, r, s_failed != 0, lane);
  // the last CTA to finish advances the call number for the next call (every
  // CTA has read it by the time it counts itself done)
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    uint32_t* done = epoch_ptr(own, a) + 1;
    if (atomicAdd(done, 1u) == gridDim.x - 1) {
      *done = 0u;
      *epoch_ptr(own, a) = epoch;
    }
  }
}

}  // namespace
}  // namespace bpkv

using namespace bpkv;

extern "C" BPKV_API size_t bpkv_peer_exchange_bytes(int world, int rows, int head_dim) {
  if (world <= 0 || world > kMaxRanks || rows <= 0 || head_dim <= 0) return 0;
  return static_cast<size_t>(data_floats(world, rows, head_dim)) * sizeof(float) + (4 * kMaxRanks + 2) * sizeof(uint32_t);
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
                                                void* out, float* lse_out, int* status, int dtype, void* stream) {
  clear_error();
  BPKV_CHECK_ARG(world >= 1 && world <= kMaxRanks && rank >= 0 && rank < world, "peer_exchange_shape:rank_%d_of_%d",
                 rank, world);
  BPKV_CHECK_ARG(rows > 0 && head_dim > 0 && head_dim % 4 == 0, "peer_exchange_shape:rows_%d_head_dim_%d", rows,
                 head_dim);
  BPKV_CHECK_ARG(part_out && part_lse && peer_bufs && out && status, "peer_exchange_shape:null_pointer");
  BPKV_CHECK_ARG(dtype == BPKV_BF16 || dtype == BPKV_F16 || dtype == BPKV_F32, "peer_exchange_shape:dtype");
  PeerArgs a;
  memset(&a, 0, sizeof(a));
  for (int r = 0; r < world; ++r) {
    BPKV_CHECK_ARG(peer_bufs[r] != nullptr && aligned16(peer_bufs[r]), "peer_exchange_shape:buffer_%d", r);
    a.bufs[r] = static_cast<float*>(peer_bufs[r]);
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
  // about 8 chunks per peer (parallel stores), at most ~16 KB of rows each
  a.rows_per_chunk = max(1, min((16384 / 4) / (head_dim + 4), (rows + 7) / 8));
  a.chunks = (rows + a.rows_per_chunk - 1) / a.rows_per_chunk;
  a.max_polls = max_polls;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int grid = max((world - 1) * a.chunks, 1);
#define BPKV_P2P(TY) peer_exchange_kernel<TY><<<grid, kSendThreads, 0, st>>>(a)
  if (dtype == BPKV_BF16) BPKV_P2P(__nv_bfloat16);
  else if (dtype == BPKV_F16) BPKV_P2P(__half);
  else BPKV_P2P(float);
#undef BPKV_P2P
  BPKV_RETURN_LAUNCH("split_kv_merge_p2p_launch");
}
