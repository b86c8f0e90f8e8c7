// 2^x evaluated on the FMA pipe (shared by the attention kernels).
#pragma once

#include <cuda_runtime.h>

namespace grx {

// 2^x on the FMA pipe, for the share of the softmax exponentials that would
// otherwise queue behind the SFU. Cody-Waite split x = n + f, n = rint(x)
// (the 1.5 * 2^23 rounding trick: FADDs only), f in [-0.5, 0.5]; 2^f from a
// degree-4 polynomial whose coefficients are a least-squares fit of 2^f at 400
// Chebyshev nodes on [-0.5, 0.5] with p(0) = 1 (relative error <= 3.2e-6 in
// fp32 Horner form, far below the bf16 rounding P goes through); 2^n is added
// to the exponent field. x is clamped at -125 so masked (-inf) scores give a
// value (~2e-38) that vanishes against the row sum.
__device__ __forceinline__ float exp2_poly(float x) {
  x = fmaxf(x, -125.0f);
  const float t = x + 12582912.0f;  // 1.5 * 2^23
  const int n = __float_as_int(t) - 0x4B400000;
  const float f = x - (t - 12582912.0f);
  float p = 0.00960039533674717f;
  p = fmaf(p, f, 0.05591689422726631f);
  p = fmaf(p, f, 0.24023719131946564f);
  p = fmaf(p, f, 0.6931219696998596f);
  p = fmaf(p, f, 1.0f);
  return __int_as_float(__float_as_int(p) + (n << 23));
}

}  // namespace grx
