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
  // Each exponential is computed once and kept in registers for the output.
  float pe[NV][EPV];
  float sum = 0.f;
#pragma unroll
  for (int v = 0; v < NV; ++v) {
    const int vi = threadIdx.x + v * kThreads;
    if (vi < nvec) {
      const T* e = reinterpret_cast<const T*>(&buf[v]);
#pragma unroll
      for (int q = 0; q < EPV; ++q) {
        pe[v][q] = expf(E<T>::f(e[q]) - mx);
        sum += pe[v][q];
      }
    }
  }
  const float inv = 1.f / block_reduce<false>(sum, red + 32);
#pragma unroll
  for (int v = 0; v < NV; ++v) {
    const int vi = threadIdx.x + v * kThreads;
    if (vi < nvec) {
      uint4 o;
      T* oe = reinterpret_cast<T*>(&o);
#pragma unroll
      for (int q = 0; q < EPV; ++q) oe[q] = E<T>::t(pe[v][q] * inv);
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

// GELU (erf form) for 16-bit outputs: x * Phi(x) with erf from Abramowitz &
// Stegun, Handbook of Mathematical Functions (1964), formula 7.1.26 (after
// Hastings): for a = |z|, t = 1 / (1 + p a),
//   1 - erf(a) = (a1 t + a2 t^2 + a3 t^3 + a4 t^4 + a5 t^5) exp(-a^2),
// absolute error <= 1.5e-7. With q = that right-hand side, 1 + erf(z) is q for
// z < 0 and 2 - q otherwise, so the far negative tail keeps its small values
// instead of cancelling. The reciprocal and 2^x are the SFU's approximate
// instructions; the result's absolute error stays below 1e-6 * |x|, far under
// a 16-bit output's rounding. In the far negative tail, where x Phi(x) is tiny,
// the relative error grows: 0.16 % at x = -5, a few % from x = -8 on (values
// below 1e-14 there). fp32 outputs keep erff.
// Phi(x) = (1 + erf(x / sqrt 2)) / 2 by the same formula.
__device__ __forceinline__ float phi_as(float x) {
  const float z = x * 0.7071067811865476f;
  const float a = fabsf(z);
  float t;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(t) : "f"(fmaf(0.3275911f, a, 1.f)));
  float poly = fmaf(1.061405429f, t, -1.453152027f);
  poly = fmaf(poly, t, 1.421413741f);
  poly = fmaf(poly, t, -0.284496736f);
  poly = fmaf(poly, t, 0.254829592f);
  poly *= t;
  float e;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(-a * a * 1.4426950408889634f));
  const float q = poly * e;
  return 0.5f * (z < 0.f ? q : 2.f - q);
}
__device__ __forceinline__ float gelu_erf_as(float x) { return x * phi_as(x); }

// The forward GELU of one element: the erf form through gelu_erf_as for
// 16-bit types, the shared epilogue activation otherwise.
template <typename T>
__device__ __forceinline__ float gelu_value(float v, int act) {
  if (sizeof(T) == 2 && act == kActGeluErf) return gelu_erf_as(v);
  return apply_act(v, act);
}

template <typename T>
__global__ void gelu_kernel(long long n, const T* x, T* y, int act, int vec) {
  constexpr int EPV = 16 / sizeof(T);
  constexpr int U = 4;  // vectors in flight per thread
  const long long stride = (long long)gridDim.x * blockDim.x;
  const long long t0 = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  if (vec) {
    const long long nv = n / EPV;
    // U vectors per thread per step: all U loads are issued before any of
    // them is used, so each thread keeps 64 bytes of reads in flight through
    // the activation arithmetic (one 16-byte vector at a time left HBM at
    // 56 % of its bandwidth).
    long long v = t0;
    for (; v + (U - 1) * stride < nv; v += U * stride) {
      uint4 b[U];
#pragma unroll
      for (int u = 0; u < U; ++u) b[u] = __ldcs(reinterpret_cast<const uint4*>(x) + v + u * stride);
#pragma unroll
      for (int u = 0; u < U; ++u) {
        T* e = reinterpret_cast<T*>(&b[u]);
        if (act == kActGeluErf) {
#pragma unroll
          for (int q = 0; q < EPV; ++q) e[q] = E<T>::t(gelu_value<T>(E<T>::f(e[q]), kActGeluErf));
        } else {
#pragma unroll
          for (int q = 0; q < EPV; ++q) e[q] = E<T>::t(gelu_value<T>(E<T>::f(e[q]), act));
        }
        __stcs(reinterpret_cast<uint4*>(y) + v + u * stride, b[u]);
      }
    }
    for (; v < nv; v += stride) {
      uint4 b = __ldcs(reinterpret_cast<const uint4*>(x) + v);
      T* e = reinterpret_cast<T*>(&b);
#pragma unroll
      for (int q = 0; q < EPV; ++q) e[q] = E<T>::t(gelu_value<T>(E<T>::f(e[q]), act));
      __stcs(reinterpret_cast<uint4*>(y) + v, b);
    }
    for (long long i = nv * EPV + t0; i < n; i += stride) y[i] = E<T>::t(gelu_value<T>(E<T>::f(x[i]), act));
  } else {
    for (long long i = t0; i < n; i += stride) y[i] = E<T>::t(gelu_value<T>(E<T>::f(x[i]), act));
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

// The same with the row's y and dy held in registers (16-byte vectors): each
// read once from HBM, dx written once.
template <typename T, int NV>
__global__ void __launch_bounds__(kThreads) softmax_bwd_vec_kernel(int cols, const T* y, long long ldy,
                                                                   const T* dy, long long lddy, T* dx,
                                                                   long long lddx) {
  constexpr int EPV = 16 / sizeof(T);
  __shared__ float red[64];
  const uint4* yr = reinterpret_cast<const uint4*>(y + (long long)blockIdx.x * ldy);
  const uint4* dr = reinterpret_cast<const uint4*>(dy + (long long)blockIdx.x * lddy);
  uint4* xr = reinterpret_cast<uint4*>(dx + (long long)blockIdx.x * lddx);
  const int nvec = cols / EPV;
  uint4 by[NV], bd[NV];
  float s = 0.f;
#pragma unroll
  for (int v = 0; v < NV; ++v) {
    const int vi = threadIdx.x + v * kThreads;
    if (vi < nvec) {
      by[v] = __ldcs(yr + vi);
      bd[v] = __ldcs(dr + vi);
    }
  }
#pragma unroll
  for (int v = 0; v < NV; ++v) {
    const int vi = threadIdx.x + v * kThreads;
    if (vi < nvec) {
      const T* ey = reinterpret_cast<const T*>(&by[v]);
      const T* ed = reinterpret_cast<const T*>(&bd[v]);
#pragma unroll
      for (int q = 0; q < EPV; ++q) s = fmaf(E<T>::f(ed[q]), E<T>::f(ey[q]), s);
    }
  }
  const float tot = block_reduce<false>(s, red);
#pragma unroll
  for (int v = 0; v < NV; ++v) {
    const int vi = threadIdx.x + v * kThreads;
    if (vi < nvec) {
      const T* ey = reinterpret_cast<const T*>(&by[v]);
      const T* ed = reinterpret_cast<const T*>(&bd[v]);
      uint4 o;
      T* eo = reinterpret_cast<T*>(&o);
#pragma unroll
      for (int q = 0; q < EPV; ++q) eo[q] = E<T>::t(E<T>::f(ey[q]) * (E<T>::f(ed[q]) - tot));
      __stcs(xr + vi, o);
    }
  }
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

// 16-bit types, erf form: Phi through phi_as and the density through the
// SFU's 2^x (relative error ~1e-6, far under the output's rounding).
template <typename T>
__device__ __forceinline__ float gelu_grad_t(float x, int act) {
  if (sizeof(T) == 2 && act == kActGeluErf) {
    float e;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(-0.5f * x * x * 1.4426950408889634f));
    return fmaf(x, 0.3989422804014327f * e, phi_as(x));
  }
  return gelu_grad(x, act);
}

// Grid-stride over 16-byte vectors of x and dy (two of each loaded per step
// before any is used) when all three pointers are 16-byte aligned; element
// by element otherwise and for the tail.
template <typename T>
__global__ void gelu_bwd_kernel(long long n, const T* x, const T* dy, T* dx,
                                int act, int vec) {
  constexpr int EPV = 16 / sizeof(T);
  const long long stride = (long long)gridDim.x * blockDim.x;
  const long long t0 = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  long long done = 0;
  if (vec) {
    const long long nv = n / EPV;
    long long v = t0;
    for (; v + stride < nv; v += 2 * stride) {
      uint4 bx[2], bd[2];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        bx[u] = __ldcs(reinterpret_cast<const uint4*>(x) + v + u * stride);
        bd[u] = __ldcs(reinterpret_cast<const uint4*>(dy) + v + u * stride);
      }
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const T* ex = reinterpret_cast<const T*>(&bx[u]);
        T* ed = reinterpret_cast<T*>(&bd[u]);
#pragma unroll
        for (int q = 0; q < EPV; ++q) ed[q] = E<T>::t(E<T>::f(ed[q]) * gelu_grad_t<T>(E<T>::f(ex[q]), act));
        __stcs(reinterpret_cast<uint4*>(dx) + v + u * stride, bd[u]);
      }
    }
    for (; v < nv; v += stride) {
      const uint4 bx = __ldcs(reinterpret_cast<const uint4*>(x) + v);
      uint4 bd = __ldcs(reinterpret_cast<const uint4*>(dy) + v);
      const T* ex = reinterpret_cast<const T*>(&bx);
      T* ed = reinterpret_cast<T*>(&bd);
#pragma unroll
      for (int q = 0; q < EPV; ++q) ed[q] = E<T>::t(E<T>::f(ed[q]) * gelu_grad_t<T>(E<T>::f(ex[q]), act));
      __stcs(reinterpret_cast<uint4*>(dx) + v, bd);
    }
    done = nv * EPV;
  }
  for (long long i = done + t0; i < n; i += stride)
    dx[i] = E<T>::t(E<T>::f(dy[i]) * gelu_grad_t<T>(E<T>::f(x[i]), act));
}

template <typename T>
cudaError_t bwd_launch(int kind, long long rows_or_n, int cols, const void* a, long long lda, const void* b,
                       long long ldb, void* c, long long ldc, int act, int num_sms, cudaStream_t s) {
  if (kind == 0) {
    constexpr int EPV = 16 / sizeof(T);
    const bool aligned = reinterpret_cast<uintptr_t>(a) % 16 == 0 && reinterpret_cast<uintptr_t>(b) % 16 == 0 &&
                         reinterpret_cast<uintptr_t>(c) % 16 == 0 && cols % EPV == 0 &&
                         (lda * (long long)sizeof(T)) % 16 == 0 && (ldb * (long long)sizeof(T)) % 16 == 0 &&
                         (ldc * (long long)sizeof(T)) % 16 == 0;
    const int nv = (cols / EPV + kThreads - 1) / kThreads;
    const T* at = static_cast<const T*>(a);
    const T* bt = static_cast<const T*>(b);
    T* ct = static_cast<T*>(c);
    const unsigned g = (unsigned)rows_or_n;
    if (aligned && nv <= 4) {
      ProfLaunch prof("softmax_bwd_vec_kernel", dim3(g), dim3(kThreads), 0, s);
      switch (nv <= 1 ? 1 : nv <= 2 ? 2 : 4) {
        case 1: softmax_bwd_vec_kernel<T, 1><<<g, kThreads, 0, s>>>(cols, at, lda, bt, ldb, ct, ldc); break;
        case 2: softmax_bwd_vec_kernel<T, 2><<<g, kThreads, 0, s>>>(cols, at, lda, bt, ldb, ct, ldc); break;
        default: softmax_bwd_vec_kernel<T, 4><<<g, kThreads, 0, s>>>(cols, at, lda, bt, ldb, ct, ldc); break;
      }
    } else {
      ProfLaunch prof("softmax_bwd_kernel", dim3(g), dim3(kThreads), 0, s);
      softmax_bwd_kernel<T><<<g, kThreads, 0, s>>>(cols, at, lda, bt, ldb, ct, ldc);
    }
  } else {
    const bool vec = reinterpret_cast<uintptr_t>(a) % 16 == 0 && reinterpret_cast<uintptr_t>(b) % 16 == 0 &&
                     reinterpret_cast<uintptr_t>(c) % 16 == 0;
    long long blocks = (rows_or_n / (vec ? 16 / (long long)sizeof(T) : 1) + kThreads - 1) / kThreads;
    if (blocks > (long long)num_sms * 8) blocks = (long long)num_sms * 8;
    if (blocks < 1) blocks = 1;
    ProfLaunch prof("gelu_bwd_kernel", dim3((unsigned)blocks), dim3(kThreads), 0, s);
    gelu_bwd_kernel<T><<<(unsigned)blocks, kThreads, 0, s>>>(rows_or_n, static_cast<const T*>(a),
                                                            static_cast<const T*>(b), static_cast<T*>(c), act,
                                                            vec ? 1 : 0);
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
