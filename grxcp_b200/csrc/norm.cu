// RMSNorm / LayerNorm forward for sm_100a (grxDNN; planned in the reference at
// docs/designs/grxcp_roadmap.md:864-876, never implemented there).
//
// HBM-bound: each row is read once into registers, reduced in fp32 with warp
// shuffles plus one shared-memory exchange, normalised from the registers and
// written once. One 256-thread CTA per row. RMSNorm moves 16-byte vectors
// (8 bf16 per thread per vector); LayerNorm, which also reads an fp32 beta,
// moves 4-element units so that every gamma / beta / x access of a warp is one
// contiguous span (with 8 elements per thread the float4 gamma/beta loads
// stride 32 bytes across the warp and double the L1 wavefronts).
// LayerNorm takes the variance as the mean of squared deviations from the
// already-reduced mean (two reductions over registers, no second read of x).
// Rows whose address, pitch or width defeat both vector paths take the scalar
// kernel below (same arithmetic, element-wise loads).
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "kernels.h"
#include "profile.h"

namespace grx {

constexpr int kNormThreads = 256;

template <typename T> struct Elem;
template <> struct Elem<float> {
  static __device__ __forceinline__ float to_f(float v) { return v; }
  static __device__ __forceinline__ float from_f(float v) { return v; }
};
template <> struct Elem<__nv_bfloat16> {
  static __device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
  static __device__ __forceinline__ __nv_bfloat16 from_f(float v) { return __float2bfloat16_rn(v); }
};
template <> struct Elem<__half> {
  static __device__ __forceinline__ float to_f(__half v) { return __half2float(v); }
  static __device__ __forceinline__ __half from_f(float v) { return __float2half_rn(v); }
};

// Sum over the CTA; every thread gets the total. Each reduction of a kernel
// gets its own `red` buffer, so one barrier per reduction suffices.
__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = lane < (int)(blockDim.x >> 5) ? red[lane] : 0.f;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
  return t;
}

// RMSNorm: NV 16-byte vectors per thread (8 bf16 each). One reduction; the
// gamma loads after it are the only other traffic.
template <typename T, int NV, bool LN>
__global__ void __launch_bounds__(kNormThreads) norm_vec_kernel(int hidden, const T* __restrict__ x, long long ldx,
                                                               const float* __restrict__ gamma,
                                                               const float* __restrict__ beta, float eps,
                                                               T* __restrict__ y, long long ldy,
                                                               float* __restrict__ mean_out,
                                                               float* __restrict__ rstd_out) {
  constexpr int EPV = 16 / sizeof(T);
  __shared__ float red[64];
  const long long row = blockIdx.x;
  const T* xr = x + row * ldx;
  T* yr = y + row * ldy;
  const int nvec = hidden / EPV;

  uint4 buf[NV];
  float sum = 0.f;
#pragma unroll
  for (int v = 0; v < NV; ++v) {
    const int vi = threadIdx.x + v * kNormThreads;
    if (vi < nvec) {
      buf[v] = __ldcs(reinterpret_cast<const uint4*>(xr) + vi);  // streamed: read exactly once
      const T* e = reinterpret_cast<const T*>(&buf[v]);
#pragma unroll
      for (int q = 0; q < EPV; ++q) {
        const float f = Elem<T>::to_f(e[q]);
        sum += LN ? f : f * f;
      }
    }
  }
  const float inv_h = 1.f / (float)hidden;
  float mu = 0.f, rstd;
  if (LN) {
    mu = block_sum(sum, red) * inv_h;
    float sq = 0.f;
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      const int vi = threadIdx.x + v * kNormThreads;
      if (vi < nvec) {
        const T* e = reinterpret_cast<const T*>(&buf[v]);
#pragma unroll
        for (int q = 0; q < EPV; ++q) {
          const float d = Elem<T>::to_f(e[q]) - mu;
          sq += d * d;
        }
      }
    }
    rstd = rsqrtf(block_sum(sq, red + 32) * inv_h + eps);
  } else {
    rstd = rsqrtf(block_sum(sum, red) * inv_h + eps);
  }
  if (threadIdx.x == 0) {
    if (mean_out) mean_out[row] = mu;
    if (rstd_out) rstd_out[row] = rstd;
  }
#pragma unroll
  for (int v = 0; v < NV; ++v) {
    const int vi = threadIdx.x + v * kNormThreads;
    if (vi < nvec) {
      const T* e = reinterpret_cast<const T*>(&buf[v]);
      uint4 o;
      T* oe = reinterpret_cast<T*>(&o);
      const int c0 = vi * EPV;
#pragma unroll
      for (int q = 0; q < EPV; q += 4) {
        const float4 g = __ldg(reinterpret_cast<const float4*>(gamma + c0 + q));
        float4 bb = make_float4(0.f, 0.f, 0.f, 0.f);
        if (LN && beta) bb = __ldg(reinterpret_cast<const float4*>(beta + c0 + q));
        const float gv[4] = {g.x, g.y, g.z, g.w}, bv[4] = {bb.x, bb.y, bb.z, bb.w};
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const float f = Elem<T>::to_f(e[q + u]);
          const float n = LN ? (f - mu) * rstd : f * rstd;
          oe[q + u] = Elem<T>::from_f(LN ? fmaf(n, gv[u], bv[u]) : n * gv[u]);
        }
      }
      __stcs(reinterpret_cast<uint4*>(yr) + vi, o);
    }
  }
}

// A "unit" is 4 consecutive elements (8 bytes of bf16/fp16, 16 of fp32), so
// the gamma / beta float4 a thread needs for a unit sits next to its
// neighbours' in the warp: every gamma, beta and x access of a warp is one
// contiguous span. NU units per thread.
template <typename T> struct Unit;
template <> struct Unit<float> { using type = uint4; };
template <> struct Unit<__nv_bfloat16> { using type = uint2; };
template <> struct Unit<__half> { using type = uint2; };

template <typename T, int NU, bool LN>
__global__ void __launch_bounds__(kNormThreads) norm_unit_kernel(int hidden, const T* __restrict__ x, long long ldx,
                                                               const float* __restrict__ gamma,
                                                               const float* __restrict__ beta, float eps,
                                                               T* __restrict__ y, long long ldy,
                                                               float* __restrict__ mean_out,
                                                               float* __restrict__ rstd_out) {
  using U = typename Unit<T>::type;
  __shared__ float red[64];
  const long long row = blockIdx.x;
  const U* xr = reinterpret_cast<const U*>(x + row * ldx);
  U* yr = reinterpret_cast<U*>(y + row * ldy);
  const int nunit = hidden / 4;

  U buf[NU];
  float sum = 0.f;
#pragma unroll
  for (int v = 0; v < NU; ++v) {
    const int ui = threadIdx.x + v * kNormThreads;
    if (ui < nunit) {
      buf[v] = __ldcs(xr + ui);  // streamed: read exactly once
      const T* e = reinterpret_cast<const T*>(&buf[v]);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float f = Elem<T>::to_f(e[q]);
        sum += LN ? f : f * f;
      }
    }
  }
  const float inv_h = 1.f / (float)hidden;
  float mu = 0.f, rstd;
  if (LN) {
    mu = block_sum(sum, red) * inv_h;
    float sq = 0.f;
#pragma unroll
    for (int v = 0; v < NU; ++v) {
      const int ui = threadIdx.x + v * kNormThreads;
      if (ui < nunit) {
        const T* e = reinterpret_cast<const T*>(&buf[v]);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float d = Elem<T>::to_f(e[q]) - mu;
          sq = fmaf(d, d, sq);
        }
      }
    }
    rstd = rsqrtf(block_sum(sq, red + 32) * inv_h + eps);
  } else {
    rstd = rsqrtf(block_sum(sum, red) * inv_h + eps);
  }
  if (threadIdx.x == 0) {
    if (mean_out) mean_out[row] = mu;
    if (rstd_out) rstd_out[row] = rstd;
  }
  const float4* g4 = reinterpret_cast<const float4*>(gamma);
  const float4* b4 = reinterpret_cast<const float4*>(beta);
#pragma unroll
  for (int v = 0; v < NU; ++v) {
    const int ui = threadIdx.x + v * kNormThreads;
    if (ui < nunit) {
      const T* e = reinterpret_cast<const T*>(&buf[v]);
      const float4 g = __ldg(g4 + ui);
      const float4 bb = (LN && beta) ? __ldg(b4 + ui) : make_float4(0.f, 0.f, 0.f, 0.f);
      const float gv[4] = {g.x, g.y, g.z, g.w}, bv[4] = {bb.x, bb.y, bb.z, bb.w};
      U o;
      T* oe = reinterpret_cast<T*>(&o);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float f = Elem<T>::to_f(e[q]);
        const float n = LN ? (f - mu) * rstd : f * rstd;
        oe[q] = Elem<T>::from_f(LN ? fmaf(n, gv[q], bv[q]) : n * gv[q]);
      }
      __stcs(yr + ui, o);
    }
  }
}

// Element-wise fallback for unaligned rows: two reads of the row (from L2).
template <typename T, bool LN>
__global__ void __launch_bounds__(kNormThreads) norm_scalar_kernel(int hidden, const T* __restrict__ x, long long ldx,
                                                                  const float* __restrict__ gamma,
                                                                  const float* __restrict__ beta, float eps,
                                                                  T* __restrict__ y, long long ldy,
                                                                  float* __restrict__ mean_out,
                                                                  float* __restrict__ rstd_out) {
  __shared__ float red[64];
  const long long row = blockIdx.x;
  const T* xr = x + row * ldx;
  T* yr = y + row * ldy;
  const float inv_h = 1.f / (float)hidden;
  float s = 0.f;
  for (int c = threadIdx.x; c < hidden; c += kNormThreads) {
    const float f = Elem<T>::to_f(xr[c]);
    s += LN ? f : f * f;
  }
  float mu = 0.f, rstd;
  if (LN) {
    mu = block_sum(s, red) * inv_h;
    float sq = 0.f;
    for (int c = threadIdx.x; c < hidden; c += kNormThreads) {
      const float d = Elem<T>::to_f(xr[c]) - mu;
      sq += d * d;
    }
    rstd = rsqrtf(block_sum(sq, red + 32) * inv_h + eps);
  } else {
    rstd = rsqrtf(block_sum(s, red) * inv_h + eps);
  }
  if (threadIdx.x == 0) {
    if (mean_out) mean_out[row] = mu;
    if (rstd_out) rstd_out[row] = rstd;
  }
  for (int c = threadIdx.x; c < hidden; c += kNormThreads) {
    const float f = Elem<T>::to_f(xr[c]);
    const float n = LN ? (f - mu) * rstd : f * rstd;
    yr[c] = Elem<T>::from_f(LN ? fmaf(n, gamma[c], beta ? beta[c] : 0.f) : n * gamma[c]);
  }
}

template <typename T, bool LN>
static cudaError_t dispatch(int rows, int hidden, const void* x, long long ldx, const float* gamma,
                            const float* beta, float eps, void* y, long long ldy, float* mean, float* rstd,
                            cudaStream_t s) {
  constexpr long long UB = 4 * sizeof(T);  // bytes of one unit
  const bool aligned = (reinterpret_cast<uintptr_t>(x) % UB == 0) && (reinterpret_cast<uintptr_t>(y) % UB == 0) &&
                       (reinterpret_cast<uintptr_t>(gamma) % 16 == 0) &&
                       (!beta || reinterpret_cast<uintptr_t>(beta) % 16 == 0) && hidden % 4 == 0 &&
                       (ldx * (long long)sizeof(T)) % UB == 0 && (ldy * (long long)sizeof(T)) % UB == 0;
  const int nunit = hidden / 4;
  const int nu = (nunit + kNormThreads - 1) / kNormThreads;
  const T* xt = static_cast<const T*>(x);
  T* yt = static_cast<T*>(y);
  constexpr int EPV = 16 / sizeof(T);
  const int nvec = hidden / EPV;
  const int nv = (nvec + kNormThreads - 1) / kNormThreads;
  const bool aligned16 = (reinterpret_cast<uintptr_t>(x) % 16 == 0) && (reinterpret_cast<uintptr_t>(y) % 16 == 0) &&
                         (reinterpret_cast<uintptr_t>(gamma) % 16 == 0) && hidden % EPV == 0 &&
                         (ldx * (long long)sizeof(T)) % 16 == 0 && (ldy * (long long)sizeof(T)) % 16 == 0;
  ProfLaunch prof(!LN && aligned16 && nv <= 8 ? "norm_vec_kernel" : (aligned && nu <= 16 ? "norm_unit_kernel" : "norm_scalar_kernel"),
                  dim3(rows), dim3(kNormThreads), 0, s);
  if (!LN && aligned16 && nv <= 8) {
#define GRX_RMS_CASE(NVV)                                                                               \
  case NVV:                                                                                             \
    norm_vec_kernel<T, NVV, false><<<rows, kNormThreads, 0, s>>>(hidden, xt, ldx, gamma, beta, eps, yt, ldy, \
                                                                  mean, rstd);                         \
    break;
    switch (nv <= 1 ? 1 : nv <= 2 ? 2 : nv <= 4 ? 4 : 8) {
      GRX_RMS_CASE(1)
      GRX_RMS_CASE(2)
      GRX_RMS_CASE(4)
      GRX_RMS_CASE(8)
    }
#undef GRX_RMS_CASE
  } else if (aligned && nu <= 16) {
#define GRX_NORM_CASE(NUU)                                                                              \
  case NUU:                                                                                             \
    norm_unit_kernel<T, NUU, LN><<<rows, kNormThreads, 0, s>>>(hidden, xt, ldx, gamma, beta, eps, yt, ldy, \
                                                               mean, rstd);                            \
    break;
    switch (nu <= 2 ? 2 : nu <= 4 ? 4 : nu <= 8 ? 8 : 16) {
      GRX_NORM_CASE(2)
      GRX_NORM_CASE(4)
      GRX_NORM_CASE(8)
      GRX_NORM_CASE(16)
    }
#undef GRX_NORM_CASE
  } else {
    norm_scalar_kernel<T, LN><<<rows, kNormThreads, 0, s>>>(hidden, xt, ldx, gamma, beta, eps, yt, ldy, mean, rstd);
  }
  return cudaGetLastError();
}

cudaError_t launch_rmsnorm(int rows, int hidden, int dtype, const void* x, long long ldx, const float* gamma,
                           float eps, void* y, long long ldy, float* rstd, cudaStream_t s) {
  switch (dtype) {
    case 0: return dispatch<float, false>(rows, hidden, x, ldx, gamma, nullptr, eps, y, ldy, nullptr, rstd, s);
    case 1: return dispatch<__nv_bfloat16, false>(rows, hidden, x, ldx, gamma, nullptr, eps, y, ldy, nullptr, rstd, s);
    case 2: return dispatch<__half, false>(rows, hidden, x, ldx, gamma, nullptr, eps, y, ldy, nullptr, rstd, s);
  }
  return cudaErrorInvalidValue;
}

cudaError_t launch_layernorm(int rows, int hidden, int dtype, const void* x, long long ldx, const float* gamma,
                             const float* beta, float eps, void* y, long long ldy, float* mean, float* rstd,
                             cudaStream_t s) {
  switch (dtype) {
    case 0: return dispatch<float, true>(rows, hidden, x, ldx, gamma, beta, eps, y, ldy, mean, rstd, s);
    case 1: return dispatch<__nv_bfloat16, true>(rows, hidden, x, ldx, gamma, beta, eps, y, ldy, mean, rstd, s);
    case 2: return dispatch<__half, true>(rows, hidden, x, ldx, gamma, beta, eps, y, ldy, mean, rstd, s);
  }
  return cudaErrorInvalidValue;
}

}  // namespace grx
