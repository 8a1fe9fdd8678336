// 2^x on the FMA pipe, for a share of the attention kernels' exponentials.
//
// The softmax phase of flash attention on sm_100a is bound by the rate of
// ex2.approx (the multi-function unit issues far fewer results per clock than
// the FMA pipe runs packed f32x2 operations), most of all at head size 64,
// where the tensor-core work per score is smallest. The kernels therefore
// compute part of their exponentials here, on the FMA pipe, and the rest with
// ex2.approx, so both pipes work in parallel.
//
// Method: range reduction x = j + f with j = round(x) and f in [-0.5, 0.5]
// (adding and subtracting 1.5 * 2^23 rounds to the nearest integer, and the
// integer is then the low mantissa bits of the sum); 2^f from a cubic whose
// coefficients were fitted for this purpose by weighted least squares
// (Lawson's iteration) to minimise the relative error on [-0.5, 0.5]: max
// relative error 7.5e-5, far below the 2^-9 resolution of the 16-bit
// probabilities it feeds; 2^j is added to the exponent field. Inputs below
// -125 (including the -inf of masked scores) give exactly 0, as their
// ex2.approx.ftz results would be negligible or flushed.
#pragma once

#include "sm100.cuh"

namespace kb {

__device__ __forceinline__ float2 ex2_fma2(float2 x) {
  constexpr float kRound = 12582912.f;  // 1.5 * 2^23
  constexpr int kRoundBits = 0x4B400000;
  const float2 xc = make_float2(fmaxf(x.x, -125.f), fmaxf(x.y, -125.f));
  const float2 r = add2(xc, make_float2(kRound, kRound));
  const float2 j = add2(r, make_float2(-kRound, -kRound));
  const float2 f = fma2(j, make_float2(-1.f, -1.f), xc);
  float2 p = fma2(f, make_float2(0.0551716648f, 0.0551716648f), make_float2(0.2426111251f, 0.2426111251f));
  p = fma2(p, f, make_float2(0.6932609677f, 0.6932609677f));
  p = fma2(p, f, make_float2(0.9999280572f, 0.9999280572f));
  const int jx = __float_as_int(r.x) - kRoundBits, jy = __float_as_int(r.y) - kRoundBits;
  float2 out = make_float2(__int_as_float(__float_as_int(p.x) + (jx << 23)),
                           __int_as_float(__float_as_int(p.y) + (jy << 23)));
  if (x.x < -125.f) out.x = 0.f;
  if (x.y < -125.f) out.y = 0.f;
  return out;
}

}  // namespace kb
