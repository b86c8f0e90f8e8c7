// Row softmax and element-wise GELU for sm_100a (grxDNN; the reference plans
// "softmax, GELU" among its grxDNN primitives at docs/designs/
// grxcp_architecture.md:594 and docs/designs/grxcp_roadmap.md:864-876, and
// implements neither).
//
// Softmax is HBM-bound like the norms: one 256-thread CTA per row, the row read
// once into registers with 16-byte loads, the max and the sum of exp(x - max)
// reduced in fp32 (warp shuffles + one smem exchange each), the result written
// once. Rows that defeat 16-byte vectors (address, pitch or width) take the
// element-wise kernel, which reads the row three times from L2.
// GELU is a grid-stride element-wise pass with 16-byte vectors where possible.
// The backward kernels (softmax: dx = y (dy - sum dy y); GELU: dx = dy GELU'(x))
// are element-wise / one-reduction passes for training.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <math.h>

#include "activation.cuh"
#include "kernels.h"
#include "profile.h"

namespace grx {

namespace {

constexpr int kThreads = 256;

template <typename T> struct E;
template <> struct E<float> {
  static __device__ __forceinline__ float f(float v) { return v; }
  static __device__ __forceinline__ float t(float v) { return v; }
};
template <> struct E<__nv_bfloat16> {
  static __device__ __forceinline__ float f(__nv_bfloat16 v) { return __bfloat162float(v); }
  static __device__ __forceinline__ __nv_bfloat16 t(float v) { return __float2bfloat16_rn(v); }
};
template <> struct E<__half> {
  static __device__ __forceinline__ float f(__half v) { return __half2float(v); }
  static __device__ __forceinline__ __half t(float v) { return __float2half_rn(v); }
};

// CTA reduction (max or sum) with a dedicated smem slot set; all threads get it.
template <bool MAX>
__device__ __forceinline__ float block_reduce(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float w = __shfl_xor_sync(0xffffffffu, v, o);
    v = MAX ? fmaxf(v, w) : v + w;
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = lane < kThreads / 32 ? red[lane] : (MAX ? -INFINITY : 0.f);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float w = __shfl_xor_sync(0xffffffffu, t, o);
    t = MAX ? fmaxf(t, w) : t + w;
  }
  return t;
}

template <typename T, int NV>
__global__ void __launch_bounds__(kThreads) softmax_vec_kernel(int cols, const T* x, long long ldx,
                                                              T* y, long long ldy) {
  constexpr int EPV = 16 / sizeof(T);
  __shared__ float red[64];
  const long long row = blockIdx.x;
  const uint4* xr = reinterpret_cast<const uint4*>(x + row * ldx);
  uint4* yr = reinterpret_cast<uint4*>(y + row * ldy);
  const int nvec = cols / EPV;
  uint4 buf[NV];
  float mx = -INFINITY;
#pragma unroll
  for (int v = 0; v < NV; ++v) {
    const int vi = threadIdx.x + v * kThreads;
    if (vi < nvec) {
      buf[v] = __ldcs(xr + vi);
      const T* e = reinterpret_cast<const T*>(&buf[v]);
#pragma unroll
      for (int q = 0; q < EPV; ++q) mx = fmaxf(mx, E<T>::f(e[q]));
    }
  }
  mx = block_reduce<true>(mx, red);
  float sum = 0.f;
#pragma unroll
  for (int v = 0; v < NV; ++v) {
    const int vi = threadIdx.x + v * kThreads;
    if (vi < nvec) {
      const T* e = reinterpret_cast<const T*>(&buf[v]);
#pragma unroll
      for (int q = 0; q < EPV; ++q) sum += expf(E<T>::f(e[q]) - mx);
    }
  }
  const float inv = 1.f / block_reduce<false>(sum, red + 32);
#pragma unroll
  for (int v = 0; v < NV; ++v) {
    const int vi = threadIdx.x + v * kThreads;
    if (vi < nvec) {
      const T* e = reinterpret_cast<const T*>(&buf[v]);
      uint4 o;
      T* oe = reinterpret_cast<T*>(&o);
#pragma unroll
      for (int q = 0; q < EPV; ++q) oe[q] = E<T>::t(expf(E<T>::f(e[q]) - mx) * inv);
      __stcs(yr + vi, o);
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(kThreads) softmax_scalar_kernel(int cols, const T* x, long long ldx,
                                                                 T* y, long long ldy) {
  __shared__ float red[64];
  const T* xr = x + (long long)blockIdx.x * ldx;
  T* yr = y + (long long)blockIdx.x * ldy;
  float mx = -INFINITY;
  for (int c = threadIdx.x; c < cols; c += kThreads) mx = fmaxf(mx, E<T>::f(xr[c]));
  mx = block_reduce<true>(mx, red);
  float sum = 0.f;
  for (int c = threadIdx.x; c < cols; c += kThreads) sum += expf(E<T>::f(xr[c]) - mx);
  const float inv = 1.f / block_reduce<false>(sum, red + 32);
  for (int c = threadIdx.x; c < cols; c += kThreads) yr[c] = E<T>::t(expf(E<T>::f(xr[c]) - mx) * inv);
}

template <typename T>
cudaError_t softmax_dispatch(int rows, int cols, const void* x, long long ldx, void* y, long long ldy,
                             cudaStream_t s) {
  constexpr int EPV = 16 / sizeof(T);
  const T* xt = static_cast<const T*>(x);
  T* yt = static_cast<T*>(y);
  const bool aligned = reinterpret_cast<uintptr_t>(x) % 16 == 0 && reinterpret_cast<uintptr_t>(y) % 16 == 0 &&
                       cols % EPV == 0 && (ldx * (long long)sizeof(T)) % 16 == 0 &&
                       (ldy * (long long)sizeof(T)) % 16 == 0;
  const int nv = (cols / EPV + kThreads - 1) / kThreads;
  ProfLaunch prof(aligned && nv <= 8 ? "softmax_vec_kernel" : "softmax_scalar_kernel", dim3(rows), dim3(kThreads), 0, s);
  if (aligned && nv <= 8) {
    switch (nv <= 1 ? 1 : nv <= 2 ? 2 : nv <= 4 ? 4 : 8) {
      case 1: softmax_vec_kernel<T, 1><<<rows, kThreads, 0, s>>>(cols, xt, ldx, yt, ldy); break;
      case 2: softmax_vec_kernel<T, 2><<<rows, kThreads, 0, s>>>(cols, xt, ldx, yt, ldy); break;
      case 4: softmax_vec_kernel<T, 4><<<rows, kThreads, 0, s>>>(cols, xt, ldx, yt, ldy); break;
      default: softmax_vec_kernel<T, 8><<<rows, kThreads, 0, s>>>(cols, xt, ldx, yt, ldy); break;
    }
  } else {
    softmax_scalar_kernel<T><<<rows, kThreads, 0, s>>>(cols, xt, ldx, yt, ldy);
  }
  return cudaGetLastError();
}

template <typename T>
__global__ void gelu_kernel(long long n, const T* x, T* y, int act, int vec) {
  constexpr int EPV = 16 / sizeof(T);
  const long long stride = (long long)gridDim.x * blockDim.x;
  const long long t0 = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  if (vec) {
    const long long nv = n / EPV;
    for (long long v = t0; v < nv; v += stride) {
      uint4 b = __ldcs(reinterpret_cast<const uint4*>(x) + v);
      T* e = reinterpret_cast<T*>(&b);
#pragma unroll
      for (int q = 0; q < EPV; ++q) e[q] = E<T>::t(apply_act(E<T>::f(e[q]), act));
      __stcs(reinterpret_cast<uint4*>(y) + v, b);
    }
    for (long long i = nv * EPV + t0; i < n; i += stride) y[i] = E<T>::t(apply_act(E<T>::f(x[i]), act));
  } else {
    for (long long i = t0; i < n; i += stride) y[i] = E<T>::t(apply_act(E<T>::f(x[i]), act));
  }
}

template <typename T>
cudaError_t gelu_dispatch(long long n, const void* x, void* y, int act, int num_sms, cudaStream_t s) {
  const bool vec = reinterpret_cast<uintptr_t>(x) % 16 == 0 && reinterpret_cast<uintptr_t>(y) % 16 == 0;
  long long blocks = (n / (vec ? 16 / (long long)sizeof(T) : 1) + kThreads - 1) / kThreads;
  const long long cap = (long long)num_sms * 8;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  ProfLaunch prof("gelu_kernel", dim3((unsigned)blocks), dim3(kThreads), 0, s);
  gelu_kernel<T><<<(unsigned)blocks, kThreads, 0, s>>>(n, static_cast<const T*>(x), static_cast<T*>(y), act,
                                                     vec ? 1 : 0);
  return cudaGetLastError();
}

// Softmax backward, one 256-thread CTA per row: dx = y * (dy - sum_c dy y),
// the row sum reduced in fp32 (three passes over the row, served from L1/L2
// after the first).
template <typename T>
__global__ void __launch_bounds__(kThreads) softmax_bwd_kernel(int cols, const T* y, long long ldy,
                                                               const T* dy, long long lddy,
                                                               T* dx, long long lddx) {
  __shared__ float red[64];
  const T* yr = y + (long long)blockIdx.x * ldy;
  const T* dr = dy + (long long)blockIdx.x * lddy;
  T* xr = dx + (long long)blockIdx.x * lddx;
  float s = 0.f;
  for (int c = threadIdx.x; c < cols; c += kThreads) s = fmaf(E<T>::f(dr[c]), E<T>::f(yr[c]), s);
  const float tot = block_reduce<false>(s, red);
  for (int c = threadIdx.x; c < cols; c += kThreads) xr[c] = E<T>::t(E<T>::f(yr[c]) * (E<T>::f(dr[c]) - tot));
}

// GELU derivative (Hendrycks & Gimpel), times dy:
//   erf form:  Phi(x) + x phi(x),  phi(x) = exp(-x^2 / 2) / sqrt(2 pi)
//   tanh form: 0.5 (1 + t) + 0.5 x (1 - t^2) sqrt(2/pi) (1 + 3 * 0.044715 x^2),
//              t = tanh(sqrt(2/pi) (x + 0.044715 x^3))
__device__ __forceinline__ float gelu_grad(float x, int act) {
  if (act == kActGeluErf) {
    const float cdf = 0.5f * (1.f + erff(x * 0.7071067811865476f));
    const float pdf = 0.3989422804014327f * expf(-0.5f * x * x);
    return fmaf(x, pdf, cdf);
  }
  const float k0 = 0.7978845608028654f, k1 = 0.044715f;
  const float t = tanhf(k0 * fmaf(k1 * x, x * x, x));
  return 0.5f * (1.f + t) + 0.5f * x * (1.f - t * t) * k0 * fmaf(3.f * k1, x * x, 1.f);
}

template <typename T>
__global__ void gelu_bwd_kernel(long long n, const T* x, const T* dy, T* dx,
                                int act) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += stride)
    dx[i] = E<T>::t(E<T>::f(dy[i]) * gelu_grad(E<T>::f(x[i]), act));
}

template <typename T>
cudaError_t bwd_launch(int kind, long long rows_or_n, int cols, const void* a, long long lda, const void* b,
                       long long ldb, void* c, long long ldc, int act, int num_sms, cudaStream_t s) {
  if (kind == 0) {
    ProfLaunch prof("softmax_bwd_kernel", dim3((unsigned)rows_or_n), dim3(kThreads), 0, s);
    softmax_bwd_kernel<T><<<(unsigned)rows_or_n, kThreads, 0, s>>>(cols, static_cast<const T*>(a), lda,
                                                                  static_cast<const T*>(b), ldb, static_cast<T*>(c),
                                                                  ldc);
  } else {
    long long blocks = (rows_or_n + kThreads - 1) / kThreads;
    if (blocks > (long long)num_sms * 16) blocks = (long long)num_sms * 16;
    if (blocks < 1) blocks = 1;
    ProfLaunch prof("gelu_bwd_kernel", dim3((unsigned)blocks), dim3(kThreads), 0, s);
    gelu_bwd_kernel<T><<<(unsigned)blocks, kThreads, 0, s>>>(rows_or_n, static_cast<const T*>(a),
                                                            static_cast<const T*>(b), static_cast<T*>(c), act);
  }
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_softmax(int rows, int cols, int dtype, const void* x, long long ldx, void* y, long long ldy,
                           cudaStream_t s) {
  switch (dtype) {
    case 0: return softmax_dispatch<float>(rows, cols, x, ldx, y, ldy, s);
    case 1: return softmax_dispatch<__nv_bfloat16>(rows, cols, x, ldx, y, ldy, s);
    case 2: return softmax_dispatch<__half>(rows, cols, x, ldx, y, ldy, s);
  }
  return cudaErrorInvalidValue;
}

cudaError_t launch_softmax_bwd(int rows, int cols, int dtype, const void* y, long long ldy, const void* dy,
                               long long lddy, void* dx, long long lddx, cudaStream_t s) {
  switch (dtype) {
    case 0: return bwd_launch<float>(0, rows, cols, y, ldy, dy, lddy, dx, lddx, 0, 0, s);
    case 1: return bwd_launch<__nv_bfloat16>(0, rows, cols, y, ldy, dy, lddy, dx, lddx, 0, 0, s);
    case 2: return bwd_launch<__half>(0, rows, cols, y, ldy, dy, lddy, dx, lddx, 0, 0, s);
  }
  return cudaErrorInvalidValue;
}

cudaError_t launch_gelu_bwd(long long n, int dtype, const void* x, const void* dy, void* dx, int act, int num_sms,
                            cudaStream_t s) {
  switch (dtype) {
    case 0: return bwd_launch<float>(1, n, 0, x, 0, dy, 0, dx, 0, act, num_sms, s);
    case 1: return bwd_launch<__nv_bfloat16>(1, n, 0, x, 0, dy, 0, dx, 0, act, num_sms, s);
    case 2: return bwd_launch<__half>(1, n, 0, x, 0, dy, 0, dx, 0, act, num_sms, s);
  }
  return cudaErrorInvalidValue;
}

cudaError_t launch_gelu(long long n, int dtype, const void* x, void* y, int act, int num_sms, cudaStream_t s) {
  switch (dtype) {
    case 0: return gelu_dispatch<float>(n, x, y, act, num_sms, s);
    case 1: return gelu_dispatch<__nv_bfloat16>(n, x, y, act, num_sms, s);
    case 2: return gelu_dispatch<__half>(n, x, y, act, num_sms, s);
  }
  return cudaErrorInvalidValue;
}

}  // namespace grx
