// 2^x on the FMA pipes (used where the MUFU's ex2, 16 a clock per SM, is
// the bottleneck and part of the exponentials can move to the FMA units).
#pragma once

#include <cuda_runtime.h>

namespace veda {

// 2^x on the FMA pipes for a pair of values: x = n + f with n = rint(x),
// f in [-1/2, 1/2]; 2^f from the degree-3 minimax polynomial fitted by
// csrc/fit_exp2_poly.py (max relative error 7.5e-5); 2^n added to the
// exponent field. Arguments below -125 (masked keys) give ~0.
__device__ __forceinline__ float2 exp2_poly2(float2 x) {
  constexpr float kRound = 12582912.0f;  // 1.5 * 2^23: rounds to integers
  x.x = fmaxf(x.x, -125.0f);
  x.y = fmaxf(x.y, -125.0f);
  const float2 t = __fadd2_rn(x, make_float2(kRound, kRound));
  const float2 n = __fadd2_rn(t, make_float2(-kRound, -kRound));
  const float2 f = __ffma2_rn(n, make_float2(-1.0f, -1.0f), x);
  float2 q = __ffma2_rn(f, make_float2(0x1.c3f76p-5f, 0x1.c3f76p-5f),
                        make_float2(0x1.f0de1ap-3f, 0x1.f0de1ap-3f));
  q = __ffma2_rn(q, f, make_float2(0x1.62f31ap-1f, 0x1.62f31ap-1f));
  q = __ffma2_rn(q, f, make_float2(0x1.fff692p-1f, 0x1.fff692p-1f));
  // The integer n sits in the low mantissa bits of t; n << 23 scales by 2^n.
  const int bx = __float_as_int(q.x) + (__float_as_int(t.x) << 23);
  const int by = __float_as_int(q.y) + (__float_as_int(t.y) << 23);
  return make_float2(__int_as_float(bx), __int_as_float(by));
}

}  // namespace veda
