// Packed fp32 pair arithmetic (the f32x2 add / sub / mul / fma of sm_100) and an
// exp2 of a pair evaluated on the FMA pipe, shared by the softmax-style kernels.
#pragma once

#include <stdint.h>

namespace bpkv {

// ---- packed fp32 pairs (f32x2 arithmetic of sm_100) ----
__device__ __forceinline__ uint64_t pk2(float a, float b) {  // a -> low half, b -> high half
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void up2(uint64_t v, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t sub2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t mul2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

// 2^x of a pair on the FMA pipe instead of the MUFU unit (which issues only 16
// exponentials per clock per SM and bounds the softmax).  Cody-Waite range
// reduction x = n + f, n = rint(x) via the 1.5*2^23 rounding constant, f in
// [-0.5, 0.5]; 2^f by a degree-5 polynomial whose coefficients were fitted by
// weighted least squares (Lawson iterations towards minimax relative error;
// max relative error 2.4e-7 evaluated in fp32, comparable to ex2.approx);
// 2^n is assembled in the exponent field from the low bits of the rounded sum.
// Valid for x < 128; x <= -127 gives exactly 0 (so -inf, masked, gives 0); NaN gives NaN.
__device__ __forceinline__ uint64_t exp2_poly2(uint64_t x2) {
  float xa, xb;
  up2(x2, xa, xb);
  xa = xa < -127.f ? -127.f : xa;  // (a NaN stays NaN)
  xb = xb < -127.f ? -127.f : xb;
  const uint64_t x = pk2(xa, xb);
  const float kRound = 12582912.f + 127.f;  // 1.5*2^23 + exponent bias
  const uint64_t t = add2(x, pk2(kRound, kRound));
  const uint64_t f = sub2(x, sub2(t, pk2(kRound, kRound)));
  uint64_t q = fma2(f, pk2(1.327647129073739e-3f, 1.327647129073739e-3f), pk2(9.675540961325169e-3f, 9.675540961325169e-3f));
  q = fma2(q, f, pk2(5.550713092088699e-2f, 5.550713092088699e-2f));
  q = fma2(q, f, pk2(2.4022120237350464e-1f, 2.4022120237350464e-1f));
  q = fma2(q, f, pk2(6.931469440460205e-1f, 6.931469440460205e-1f));
  q = fma2(q, f, pk2(1.0000001192092896f, 1.0000001192092896f));
  float ta, tb;
  up2(t, ta, tb);
  const uint64_t scale = pk2(__uint_as_float(__float_as_uint(ta) << 23), __uint_as_float(__float_as_uint(tb) << 23));
  return mul2(q, scale);
}

}  // namespace bpkv
