// Element-wise activations shared by the GEMM epilogue and grxDNN.
#pragma once

#include <cuda_runtime.h>

namespace grx {

enum : int { kActNone = 0, kActRelu = 1, kActGeluTanh = 2, kActGeluErf = 3 };

// GELU (Hendrycks & Gimpel): x * Phi(x) with the Gaussian CDF written through
// erf, or its tanh approximation 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3))).
__device__ __forceinline__ float apply_act(float v, int act) {
  switch (act) {
    case kActRelu: return fmaxf(v, 0.f);
    case kActGeluTanh: {
      const float u = 0.7978845608028654f * fmaf(0.044715f * v, v * v, v);
      return 0.5f * v * (1.f + tanhf(u));
    }
    case kActGeluErf: return 0.5f * v * (1.f + erff(v * 0.7071067811865476f));
    default: return v;
  }
}

}  // namespace grx
