// Exchange-buffer layout and word format of the NVLink split-KV merge.
//
// Every rank owns one exchange buffer (cudaMalloc'd by this library, exported
// to the other processes by CUDA IPC and mapped there once):
//   uint4  word[2][world][rows][D/2 + 1]   (parity, source rank, row)
//   uint32 epoch, done                     (local: calls completed, CTAs done)
// A 16-byte word is two 64-bit halves; each half is (fp32 value bits) | (call
// number << 32).  The row's first D/2 words hold out[2j] and out[2j+1], the last
// one holds lse and 0.  Words are stored and loaded as .v2.u64 vectors: the
// memory model makes each 64-bit element of a vector access single-copy atomic
// (a vector access gives no atomicity or order across its elements), so a reader
// that sees call number e in a half has that half's value of call e, whatever
// the other half holds.  So there is no fence, counter or separate flag: the
// exchange costs one NVLink store latency.  Call number e (kept in device memory,
// so the kernels can be captured in a CUDA graph and replayed) uses parity e & 1:
// a peer may already write call e+1 while this rank still merges e; e+2 cannot
// start before this rank has finished e (the peer's call e+1 needed this rank's
// e+1 words, which come after e).  A stale word holds an older call number, so
// nothing is ever reset.
#pragma once

#include "common.cuh"

namespace bpkv {
namespace peer {

constexpr int kMaxRanks = 8;

__host__ __device__ inline int64_t row_words(int D) { return D / 2 + 1; }
__host__ __device__ inline int64_t data_words(int world, int rows, int D) {
  return 2LL * world * rows * row_words(D);
}
__host__ inline size_t exchange_bytes(int world, int rows, int D) {
  return static_cast<size_t>(data_words(world, rows, D)) * sizeof(uint4) + 4 * sizeof(uint32_t);
}
__device__ inline uint4* row_ptr(uint4* buf, int world, int rows, int D, int par, int src, int r) {
  return buf + ((static_cast<int64_t>(par) * world + src) * rows + r) * row_words(D);
}
__device__ inline uint32_t* epoch_ptr(uint4* buf, int world, int rows, int D) {
  return reinterpret_cast<uint32_t*>(buf + data_words(world, rows, D));
}

__device__ __forceinline__ void st_word(uint4* p, float x0, float x1, uint32_t epoch) {
  const uint64_t a = (static_cast<uint64_t>(epoch) << 32) | __float_as_uint(x0);
  const uint64_t b = (static_cast<uint64_t>(epoch) << 32) | __float_as_uint(x1);
  asm volatile("st.relaxed.sys.global.v2.u64 [%0], {%1,%2};\n" ::"l"(p), "l"(a), "l"(b) : "memory");
}
__device__ __forceinline__ void ld_word(const uint4* p, uint64_t& a, uint64_t& b) {
  asm volatile("ld.relaxed.sys.global.v2.u64 {%0,%1}, [%2];\n" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}
__device__ __forceinline__ uint64_t now_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Spin until both halves of the word carry `epoch`; bounded by the poll budget
// and by 4 s from t0.  Returns false (values undefined) when it ran out.
__device__ __forceinline__ bool wait_word(const uint4* p, uint32_t epoch, uint32_t& polls, uint32_t max_polls,
                                          uint64_t t0, float& x0, float& x1) {
  for (;;) {
    uint64_t a, b;
    ld_word(p, a, b);
    if (static_cast<uint32_t>(a >> 32) == epoch && static_cast<uint32_t>(b >> 32) == epoch) {
      x0 = __uint_as_float(static_cast<uint32_t>(a));
      x1 = __uint_as_float(static_cast<uint32_t>(b));
      return true;
    }
    if (++polls > max_polls || ((polls & 63u) == 0u && now_ns() - t0 > 4000000000ull)) return false;
  }
}

// The last CTA of a call to count itself done advances the call number (every CTA
// has read it by then).  Called by thread 0 after a __syncthreads.
__device__ __forceinline__ void finish_call(uint4* own, int world, int rows, int D, uint32_t epoch) {
  __threadfence();
  uint32_t* ep = epoch_ptr(own, world, rows, D);
  if (atomicAdd(ep + 1, 1u) == gridDim.x * gridDim.y - 1) {
    ep[1] = 0u;
    ep[0] = epoch;
  }
}

}  // namespace peer
}  // namespace bpkv
