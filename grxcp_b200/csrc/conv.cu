// grxDNN conv2d fallback and 2-D pooling for sm_100a. The reference plans
// "conv2d (implicit GEMM), pooling" for grxDNN (docs/designs/
// grxcp_architecture.md:594, docs/designs/grxcp_roadmap.md:864) and
// implements neither.
//
// conv2d's main path is the tcgen05 implicit GEMM in gemm_tc.cu (NHWC input
// with a channel count that is a multiple of 64). Everything else -- a first
// layer with 3 channels, odd channel counts, fp32 tensors -- runs the direct
// kernel here: one thread per output element (n, p, q, k), fp32 accumulation
// over the filter taps and channels. It is correct for every shape the API
// accepts and is not meant to be fast.
//
// Pooling (NHWC, max or average with or without padding in the divisor) is
// HBM-bound: one thread per (output pixel, channel), consecutive threads on
// consecutive channels, so every window read is coalesced across a warp.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <math.h>

#include "activation.cuh"
#include "kernels.h"
#include "profile.h"

namespace grx {

namespace {

template <typename T> struct Cv;
template <> struct Cv<float> {
  static __device__ __forceinline__ float f(float v) { return v; }
  static __device__ __forceinline__ float t(float v) { return v; }
};
template <> struct Cv<__nv_bfloat16> {
  static __device__ __forceinline__ float f(__nv_bfloat16 v) { return __bfloat162float(v); }
  static __device__ __forceinline__ __nv_bfloat16 t(float v) { return __float2bfloat16_rn(v); }
};
template <> struct Cv<__half> {
  static __device__ __forceinline__ float f(__half v) { return __half2float(v); }
  static __device__ __forceinline__ __half t(float v) { return __float2half_rn(v); }
};

template <typename TI, typename TO>
__global__ void conv2d_direct_kernel(ConvArgs a, const TI* __restrict__ x, const TI* __restrict__ w,
                                     TO* __restrict__ y) {
  const long long total = (long long)a.n * a.p * a.q * a.k;
  for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total;
       e += (long long)gridDim.x * blockDim.x) {
    const int k = (int)(e % a.k);
    long long t = e / a.k;
    const int q = (int)(t % a.q);
    t /= a.q;
    const int p = (int)(t % a.p);
    const int n = (int)(t / a.p);
    float acc = 0.f;
    for (int r = 0; r < a.r; ++r) {
      const int hh = p * a.stride_h - a.pad_h + r * a.dil_h;
      if (hh < 0 || hh >= a.h) continue;
      for (int s = 0; s < a.s; ++s) {
        const int ww = q * a.stride_w - a.pad_w + s * a.dil_w;
        if (ww < 0 || ww >= a.w) continue;
        const TI* xr = x + (((long long)n * a.h + hh) * a.w + ww) * a.c;
        const TI* wr = w + (((long long)k * a.r + r) * a.s + s) * a.c;
        for (int c = 0; c < a.c; ++c) acc = fmaf(Cv<TI>::f(xr[c]), Cv<TI>::f(wr[c]), acc);
      }
    }
    float v = __fmul_rn(a.alpha, acc);
    if (a.beta != 0.f) v = __fadd_rn(v, __fmul_rn(a.beta, Cv<TO>::f(y[e])));
    if (a.bias) v = __fadd_rn(v, a.bias[k]);
    y[e] = Cv<TO>::t(apply_act(v, a.act));
  }
}

template <typename T>
__global__ void pool2d_kernel(PoolArgs a, const T* __restrict__ x, T* __restrict__ y) {
  const long long total = (long long)a.n * a.p * a.q * a.c;
  for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total;
       e += (long long)gridDim.x * blockDim.x) {
    const int c = (int)(e % a.c);
    long long t = e / a.c;
    const int q = (int)(t % a.q);
    t /= a.q;
    const int p = (int)(t % a.p);
    const int n = (int)(t / a.p);
    float m = -INFINITY, sum = 0.f;
    int cnt = 0;
    for (int r = 0; r < a.r; ++r) {
      const int hh = p * a.stride_h - a.pad_h + r;
      if (hh < 0 || hh >= a.h) continue;
      for (int s = 0; s < a.s; ++s) {
        const int ww = q * a.stride_w - a.pad_w + s;
        if (ww < 0 || ww >= a.w) continue;
        const float v = Cv<T>::f(x[(((long long)n * a.h + hh) * a.w + ww) * a.c + c]);
        m = fmaxf(m, v);
        sum += v;
        ++cnt;
      }
    }
    float out;
    if (a.mode == 0) out = cnt ? m : 0.f;  // a window entirely in the padding yields 0
    else if (a.mode == 1) out = sum / (float)(a.r * a.s);
    else out = cnt ? sum / (float)cnt : 0.f;
    y[e] = Cv<T>::t(out);
  }
}

unsigned grid_for(long long total, int num_sms) {
  long long b = (total + 255) / 256;
  const long long cap = (long long)num_sms * 16;
  if (b > cap) b = cap;
  return (unsigned)(b < 1 ? 1 : b);
}

}  // namespace

cudaError_t launch_conv2d_direct(const ConvArgs& a, int num_sms, cudaStream_t s) {
  const long long total = (long long)a.n * a.p * a.q * a.k;
  const unsigned g = grid_for(total, num_sms);
  ProfLaunch prof("conv2d_direct_kernel", dim3(g), dim3(256), 0, s);
  switch (a.in_dtype * 4 + a.out_dtype) {
    case 1 * 4 + 1:
      conv2d_direct_kernel<__nv_bfloat16, __nv_bfloat16><<<g, 256, 0, s>>>(
          a, static_cast<const __nv_bfloat16*>(a.x), static_cast<const __nv_bfloat16*>(a.filt),
          static_cast<__nv_bfloat16*>(a.y));
      break;
    case 1 * 4 + 0:
      conv2d_direct_kernel<__nv_bfloat16, float><<<g, 256, 0, s>>>(
          a, static_cast<const __nv_bfloat16*>(a.x), static_cast<const __nv_bfloat16*>(a.filt), static_cast<float*>(a.y));
      break;
    case 0 * 4 + 0:
      conv2d_direct_kernel<float, float><<<g, 256, 0, s>>>(a, static_cast<const float*>(a.x),
                                                           static_cast<const float*>(a.filt), static_cast<float*>(a.y));
      break;
    default: return cudaErrorNotSupported;
  }
  return cudaGetLastError();
}

// 16-bit pooling with the channel count a multiple of 8 and 16-byte aligned
// tensors: one thread per (output pixel, 8 consecutive channels), every
// window tap one 16-byte load (a warp covers 512 contiguous bytes of a row of
// the window). Same arithmetic per channel as pool2d_kernel.
template <typename T>
__global__ void pool2d_vec_kernel(PoolArgs a, const T* __restrict__ x, T* __restrict__ y) {
  const int cv = a.c / 8;
  const long long total = (long long)a.n * a.p * a.q * cv;
  for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total;
       e += (long long)gridDim.x * blockDim.x) {
    const int c8 = (int)(e % cv);
    long long t = e / cv;
    const int q = (int)(t % a.q);
    t /= a.q;
    const int p = (int)(t % a.p);
    const int n = (int)(t / a.p);
    float m[8], sum[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      m[i] = -INFINITY;
      sum[i] = 0.f;
    }
    int cnt = 0;
    auto tap = [&](const uint4& b) {
      const T* ev = reinterpret_cast<const T*>(&b);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float v = Cv<T>::f(ev[i]);
        m[i] = fmaxf(m[i], v);
        sum[i] += v;
      }
      ++cnt;
    };
    if (a.r * a.s <= 9) {
      // Windows of up to 9 taps: every tap's load is issued before the first
      // is used, so the taps' latencies overlap; taps are visited in the
      // same row-major order as below.
      uint4 b[9];
      bool ok[9];
#pragma unroll
      for (int i = 0; i < 9; ++i) {
        const int r = i / a.s, s2 = i - (i / a.s) * a.s;
        const int hh = p * a.stride_h - a.pad_h + r, ww = q * a.stride_w - a.pad_w + s2;
        ok[i] = i < a.r * a.s && hh >= 0 && hh < a.h && ww >= 0 && ww < a.w;
        if (ok[i])
          b[i] = __ldg(reinterpret_cast<const uint4*>(x + (((long long)n * a.h + hh) * a.w + ww) * a.c) + c8);
      }
#pragma unroll
      for (int i = 0; i < 9; ++i)
        if (ok[i]) tap(b[i]);
    } else {
      for (int r = 0; r < a.r; ++r) {
        const int hh = p * a.stride_h - a.pad_h + r;
        if (hh < 0 || hh >= a.h) continue;
        for (int s2 = 0; s2 < a.s; ++s2) {
          const int ww = q * a.stride_w - a.pad_w + s2;
          if (ww < 0 || ww >= a.w) continue;
          tap(__ldg(reinterpret_cast<const uint4*>(x + (((long long)n * a.h + hh) * a.w + ww) * a.c) + c8));
        }
      }
    }
    uint4 o;
    T* eo = reinterpret_cast<T*>(&o);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      float out;
      if (a.mode == 0) out = cnt ? m[i] : 0.f;  // a window entirely in the padding yields 0
      else if (a.mode == 1) out = sum[i] / (float)(a.r * a.s);
      else out = cnt ? sum[i] / (float)cnt : 0.f;
      eo[i] = Cv<T>::t(out);
    }
    reinterpret_cast<uint4*>(y)[e] = o;
  }
}

cudaError_t launch_pool2d(const PoolArgs& a, int num_sms, cudaStream_t s) {
  const bool vec = a.dtype != 0 && a.c % 8 == 0 && reinterpret_cast<uintptr_t>(a.x) % 16 == 0 &&
                   reinterpret_cast<uintptr_t>(a.y) % 16 == 0;
  if (vec) {
    const unsigned g = grid_for((long long)a.n * a.p * a.q * (a.c / 8), num_sms);
    ProfLaunch prof("pool2d_vec_kernel", dim3(g), dim3(256), 0, s);
    if (a.dtype == 1)
      pool2d_vec_kernel<__nv_bfloat16><<<g, 256, 0, s>>>(a, static_cast<const __nv_bfloat16*>(a.x),
                                                          static_cast<__nv_bfloat16*>(a.y));
    else if (a.dtype == 2)
      pool2d_vec_kernel<__half><<<g, 256, 0, s>>>(a, static_cast<const __half*>(a.x), static_cast<__half*>(a.y));
    else
      return cudaErrorNotSupported;
    return cudaGetLastError();
  }
  const long long total = (long long)a.n * a.p * a.q * a.c;
  const unsigned g = grid_for(total, num_sms);
  ProfLaunch prof("pool2d_kernel", dim3(g), dim3(256), 0, s);
  switch (a.dtype) {
    case 0: pool2d_kernel<float><<<g, 256, 0, s>>>(a, static_cast<const float*>(a.x), static_cast<float*>(a.y)); break;
    case 1:
      pool2d_kernel<__nv_bfloat16><<<g, 256, 0, s>>>(a, static_cast<const __nv_bfloat16*>(a.x),
                                                      static_cast<__nv_bfloat16*>(a.y));
      break;
    case 2:
      pool2d_kernel<__half><<<g, 256, 0, s>>>(a, static_cast<const __half*>(a.x), static_cast<__half*>(a.y));
      break;
    default: return cudaErrorNotSupported;
  }
  return cudaGetLastError();
}

}  // namespace grx
