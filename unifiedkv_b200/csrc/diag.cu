// Diagnostics: a throughput probe of the special-function unit's exp2
// (ex2.approx.ftz.f32, the instruction the scoring and softmax kernels use),
// so that "bound by exponentials" is a measured fraction rather than a guess.
//
// Every thread runs kChains independent dependency chains of `iters` exp2 each
// (x <- exp2(x) * c - d keeps the argument in range and the chains alive); one
// FMA per exp2 rides along on another pipe.  The caller times the launch with
// CUDA events and divides blocks * threads * kChains * iters by the time.
#include "common.cuh"

namespace bpkv {
namespace {

constexpr int kChains = 8;

__global__ void __launch_bounds__(256) exp2_rate_kernel(int iters, float* sink) {
  float x[kChains];
#pragma unroll
  for (int c = 0; c < kChains; ++c) x[c] = -0.001f * static_cast<float>(threadIdx.x + c);
  for (int i = 0; i < iters; ++i) {
#pragma unroll
    for (int c = 0; c < kChains; ++c) x[c] = fast_exp2(x[c]) * 0.5f - 1.0f;  // stays in [-1, -0.5]
  }
  float s = 0.f;
#pragma unroll
  for (int c = 0; c < kChains; ++c) s += x[c];
  if (s == 1234.5f) *sink = s;  // never true; keeps the work
}

}  // namespace
}  // namespace bpkv

using namespace bpkv;

extern "C" BPKV_API int bpkv_debug_exp2_rate(int blocks, int iters, float* sink, void* stream) {
  clear_error();
  BPKV_CHECK_ARG(blocks > 0 && iters > 0 && sink != nullptr, "debug_exp2_rate:args");
  exp2_rate_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(iters, sink);
  BPKV_RETURN_LAUNCH("debug_exp2_rate_launch");
}

extern "C" BPKV_API long long bpkv_debug_exp2_count(int blocks, int iters) {
  return static_cast<long long>(blocks) * 256LL * kChains * static_cast<long long>(iters);
}
