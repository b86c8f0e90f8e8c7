// RMSNorm / LayerNorm backward for sm_100a (grxDNN). Neither exists in the
// reference (its grxDNN is planned only, docs/designs/grxcp_roadmap.md:
// 860-876); they are the step before the forward kernels of norm.cu in a
// training pass. With r = rstd of the row, H = hidden, g = gamma:
//   RMSNorm:   dx = r g dy - x r^3 (sum_c dy g x) / H,   dgamma = sum_rows dy x r
//   LayerNorm: xh = (x - mu) r,  dxh = dy g,
//              dx = r (dxh - (sum_c dxh) / H - xh (sum_c dxh xh) / H),
//              dgamma = sum_rows dy xh,  dbeta = sum_rows dy
// Statistics come from the forward pass (rstd, and mean for LayerNorm) or,
// when the caller passes none, are recomputed from x exactly as the forward
// kernels compute them.
//
// HBM-bound: x and dy are read once and dx written once (6 bytes per bf16
// element). Dense path: a persistent grid of (SMs x resident CTAs) walks the
// rows; each 256-thread CTA holds one row in registers (16-byte vectors),
// reduces the row sums with shuffles plus one shared-memory exchange, writes
// dx, and keeps its columns' dgamma / dbeta partial sums in registers across
// all its rows. At the end each CTA writes one partial row to scratch and a
// column kernel sums the partial rows in CTA order (deterministic, no
// atomics). Other shapes (unaligned rows, hidden not a multiple of 8 or
// above 8192) take a scalar row kernel plus a column kernel that re-reads x
// and dy.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdlib.h>

#include "kernels.h"
#include "profile.h"

namespace grx {

namespace {

constexpr int kThreads = 256;

template <typename T> struct Ev;
template <> struct Ev<float> {
  static __device__ __forceinline__ float f(float v) { return v; }
  static __device__ __forceinline__ float t(float v) { return v; }
};
template <> struct Ev<__nv_bfloat16> {
  static __device__ __forceinline__ float f(__nv_bfloat16 v) { return __bfloat162float(v); }
  static __device__ __forceinline__ __nv_bfloat16 t(float v) { return __float2bfloat16_rn(v); }
};
template <> struct Ev<__half> {
  static __device__ __forceinline__ float f(__half v) { return __half2float(v); }
  static __device__ __forceinline__ __half t(float v) { return __float2half_rn(v); }
};

// CTA sums of two values; every thread gets both. `red` holds 2 x 8 floats
// and must not be reused before another barrier has passed.
__device__ __forceinline__ float2 block_sum2(float a, float b, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    a += __shfl_xor_sync(0xffffffffu, a, o);
    b += __shfl_xor_sync(0xffffffffu, b, o);
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    red[warp] = a;
    red[8 + warp] = b;
  }
  __syncthreads();
  float ta = lane < kThreads / 32 ? red[lane] : 0.f;
  float tb = lane < kThreads / 32 ? red[8 + lane] : 0.f;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    ta += __shfl_xor_sync(0xffffffffu, ta, o);
    tb += __shfl_xor_sync(0xffffffffu, tb, o);
  }
  return make_float2(ta, tb);
}

// Bulk prefetch of `bytes` (a multiple of 16, 16-byte aligned) into L2.
__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// PF: at the top of each row, one thread asks L2 for this CTA's next row of x
// and dy (bulk prefetch). The registers hold one row per CTA, so without it a
// CTA has no reads in flight from its reduction until its next row's loads;
// the prefetch keeps DRAM busy across that gap and the next row's loads then
// hit L2. Measured at [65536, 8192] bf16 with saved statistics: LayerNorm
// 656 -> 566 us (4.9 -> 5.7 TB/s), RMSNorm 603 -> 526 us (5.3 -> 6.1 TB/s).
// GRX_NORM_BWD_NO_PREFETCH=1 turns it off.
template <typename T, int NV, bool LN, bool PF = false>
__global__ void __launch_bounds__(kThreads) norm_bwd_vec_kernel(
    int rows, int hidden, const T* __restrict__ x, long long ldx, const T* __restrict__ dy, long long lddy,
    const float* __restrict__ gamma, const float* __restrict__ mean_in, const float* __restrict__ rstd_in, float eps,
    T* __restrict__ dx, long long lddx, float* __restrict__ part) {
  // RMSNorm (80 registers, 3 CTAs per SM) gains from loading the next row
  // during the store tail (5.13 -> 5.45 TB/s at [65536, 8192] bf16);
  // LayerNorm (128 registers, 2 CTAs per SM) loses (4.83 -> 3.33 TB/s), so it
  // loads each row at the top of its iteration.
  constexpr bool pipe = !LN;
  constexpr int EPV = 16 / sizeof(T);
  __shared__ float red[2][3][16];
  const int nvec = hidden / EPV;
  const float inv_h = 1.f / (float)hidden;
  float acc_g[NV][EPV], acc_b[NV][EPV];
#pragma unroll
  for (int v = 0; v < NV; ++v)
#pragma unroll
    for (int q = 0; q < EPV; ++q) acc_g[v][q] = acc_b[v][q] = 0.f;

  // With `pipe`, two rows are in flight in the same registers: as soon as
  // vector v of row r has been written out, vector v of this CTA's next row is
  // loaded into its registers, so the next row's loads overlap this row's
  // store tail.
  uint4 bx[NV], bd[NV];
  if (blockIdx.x < rows) {
    const T* xr = x + (long long)blockIdx.x * ldx;
    const T* dyr = dy + (long long)blockIdx.x * lddy;
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      const int vi = threadIdx.x + v * kThreads;
      if (vi < nvec) {
        bx[v] = __ldcs(reinterpret_cast<const uint4*>(xr) + vi);
        bd[v] = __ldcs(reinterpret_cast<const uint4*>(dyr) + vi);
      }
    }
  }
  int parity = 0;
  for (int row = blockIdx.x; row < rows; row += gridDim.x, parity ^= 1) {
    const int next = row + gridDim.x;
    if constexpr (!pipe) if (row != blockIdx.x) {
#pragma unroll
      for (int v = 0; v < NV; ++v) {
        const int vi = threadIdx.x + v * kThreads;
        if (vi < nvec) {
          bx[v] = __ldcs(reinterpret_cast<const uint4*>(x + (long long)row * ldx) + vi);
          bd[v] = __ldcs(reinterpret_cast<const uint4*>(dy + (long long)row * lddy) + vi);
        }
      }
    }
    const T* xn = x + (long long)next * ldx;
    const T* dyn = dy + (long long)next * lddy;
    if constexpr (PF) {
      if (threadIdx.x == 0 && next < rows) {
        prefetch_l2(xn, (uint32_t)(nvec * 16));
        prefetch_l2(dyn, (uint32_t)(nvec * 16));
      }
    }
    // Row statistics: saved ones, or the forward kernels' own recipe.
    float mu = 0.f, r;
    if (rstd_in) {
      r = rstd_in[row];
      if (LN) mu = mean_in[row];
    } else {
      float s1 = 0.f;
#pragma unroll
      for (int v = 0; v < NV; ++v)
        if (threadIdx.x + v * kThreads < nvec) {
          const T* e = reinterpret_cast<const T*>(&bx[v]);
#pragma unroll
          for (int q = 0; q < EPV; ++q) {
            const float f = Ev<T>::f(e[q]);
            s1 += LN ? f : f * f;
          }
        }
      const float tot = block_sum2(s1, 0.f, red[parity][0]).x;
      if (LN) {
        mu = tot * inv_h;
        float s2 = 0.f;
#pragma unroll
        for (int v = 0; v < NV; ++v)
          if (threadIdx.x + v * kThreads < nvec) {
            const T* e = reinterpret_cast<const T*>(&bx[v]);
#pragma unroll
            for (int q = 0; q < EPV; ++q) {
              const float d = Ev<T>::f(e[q]) - mu;
              s2 += d * d;
            }
          }
        r = rsqrtf(block_sum2(s2, 0.f, red[parity][1]).x * inv_h + eps);
      } else {
        r = rsqrtf(tot * inv_h + eps);
      }
    }
    // Row sums of the gradient terms, and this row's parameter-gradient terms.
    float s_a = 0.f, s_b = 0.f;
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      const int vi = threadIdx.x + v * kThreads;
      if (vi < nvec) {
        const T* ex = reinterpret_cast<const T*>(&bx[v]);
        const T* ed = reinterpret_cast<const T*>(&bd[v]);
        const float4* gp = reinterpret_cast<const float4*>(gamma + vi * EPV);
#pragma unroll
        for (int h = 0; h < EPV / 4; ++h) {
          const float4 g4 = __ldg(gp + h);
          const float gg[4] = {g4.x, g4.y, g4.z, g4.w};
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float xf = Ev<T>::f(ex[4 * h + q]), df = Ev<T>::f(ed[4 * h + q]);
            const float dxh = df * gg[q];
            if (LN) {
              const float xh = (xf - mu) * r;
              s_a += dxh;
              s_b += dxh * xh;
              acc_g[v][4 * h + q] += df * xh;
              acc_b[v][4 * h + q] += df;
            } else {
              s_a += dxh * xf;
              acc_g[v][4 * h + q] += df * xf * r;
            }
          }
        }
      }
    }
    const float2 s = block_sum2(s_a, s_b, red[parity][2]);
    const float c1 = LN ? s.x * inv_h : 0.f;
    const float c2 = LN ? s.y * inv_h : r * r * r * s.x * inv_h;
    T* dxr = dx + (long long)row * lddx;
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      const int vi = threadIdx.x + v * kThreads;
      if (vi < nvec) {
        const T* ex = reinterpret_cast<const T*>(&bx[v]);
        const T* ed = reinterpret_cast<const T*>(&bd[v]);
        const float4* gp = reinterpret_cast<const float4*>(gamma + vi * EPV);
        uint4 o;
        T* eo = reinterpret_cast<T*>(&o);
#pragma unroll
        for (int h = 0; h < EPV / 4; ++h) {
          const float4 g4 = __ldg(gp + h);
          const float gg[4] = {g4.x, g4.y, g4.z, g4.w};
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float xf = Ev<T>::f(ex[4 * h + q]), df = Ev<T>::f(ed[4 * h + q]);
            const float dxh = df * gg[q];
            eo[4 * h + q] = Ev<T>::t(LN ? r * (dxh - c1 - (xf - mu) * r * c2) : r * dxh - xf * c2);
          }
        }
        __stcs(reinterpret_cast<uint4*>(dxr) + vi, o);
        if (pipe && next < rows) {
          bx[v] = __ldcs(reinterpret_cast<const uint4*>(xn) + vi);
          bd[v] = __ldcs(reinterpret_cast<const uint4*>(dyn) + vi);
        }
      }
    }
  }
  if (part) {
    float* pg = part + (size_t)blockIdx.x * hidden;
    float* pb = part + ((size_t)gridDim.x + blockIdx.x) * hidden;
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      const int vi = threadIdx.x + v * kThreads;
      if (vi < nvec) {
#pragma unroll
        for (int h = 0; h < EPV / 4; ++h) {
          reinterpret_cast<float4*>(pg + vi * EPV)[h] =
              make_float4(acc_g[v][4 * h], acc_g[v][4 * h + 1], acc_g[v][4 * h + 2], acc_g[v][4 * h + 3]);
          if (LN)
            reinterpret_cast<float4*>(pb + vi * EPV)[h] =
                make_float4(acc_b[v][4 * h], acc_b[v][4 * h + 1], acc_b[v][4 * h + 2], acc_b[v][4 * h + 3]);
        }
      }
    }
  }
}

// dgamma[c] (and dbeta[c]) = sum over the G partial rows. A 256-thread CTA
// covers 32 columns: its 8 warps each sum a contiguous range of the partial
// rows (lane = column, coalesced), then warp 0 adds the 8 range sums in range
// order, so the result does not depend on scheduling. blockIdx.y picks dgamma
// (0) or dbeta (1). One thread per column walking all G rows took 37-45 us at
// [65536, 8192] (G = 296..444).
constexpr int kSumCols = 32, kSumWarps = 8;
__global__ void __launch_bounds__(kSumCols * kSumWarps) norm_bwd_sum_parts_kernel(int hidden, int g,
                                                                                 const float* __restrict__ part,
                                                                                 float* dgamma, float* dbeta) {
  __shared__ float acc[kSumWarps][kSumCols];
  float* out = blockIdx.y == 0 ? dgamma : dbeta;
  if (out == nullptr) return;  // uniform over the CTA
  const float* base = part + (blockIdx.y == 0 ? 0 : (size_t)g * hidden);
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int c = blockIdx.x * kSumCols + lane;
  const int i0 = (int)((long long)g * w / kSumWarps), i1 = (int)((long long)g * (w + 1) / kSumWarps);
  float s = 0.f;
  if (c < hidden)
    for (int i = i0; i < i1; ++i) s += base[(size_t)i * hidden + c];
  acc[w][lane] = s;
  __syncthreads();
  if (w == 0 && c < hidden) {
    float t = acc[0][lane];
#pragma unroll
    for (int k = 1; k < kSumWarps; ++k) t += acc[k][lane];
    out[c] = t;
  }
}

// Scalar fallback, one CTA per row: dx, plus the row statistics into
// mean_ws / rstd_ws for the column kernel when the caller passed none.
template <typename T, bool LN>
__global__ void __launch_bounds__(kThreads) norm_bwd_row_scalar_kernel(
    int hidden, const T* __restrict__ x, long long ldx, const T* __restrict__ dy, long long lddy,
    const float* __restrict__ gamma, const float* __restrict__ mean_in, const float* __restrict__ rstd_in, float eps,
    T* __restrict__ dx, long long lddx, float* mean_ws, float* rstd_ws) {
  __shared__ float red[3][16];
  const long long row = blockIdx.x;
  const T* xr = x + row * ldx;
  const T* dyr = dy + row * lddy;
  const float inv_h = 1.f / (float)hidden;
  float mu = 0.f, r;
  if (rstd_in) {
    r = rstd_in[row];
    if (LN) mu = mean_in[row];
  } else {
    float s1 = 0.f;
    for (int c = threadIdx.x; c < hidden; c += kThreads) {
      const float f = Ev<T>::f(xr[c]);
      s1 += LN ? f : f * f;
    }
    const float tot = block_sum2(s1, 0.f, red[0]).x;
    if (LN) {
      mu = tot * inv_h;
      float s2 = 0.f;
      for (int c = threadIdx.x; c < hidden; c += kThreads) {
        const float d = Ev<T>::f(xr[c]) - mu;
        s2 += d * d;
      }
      r = rsqrtf(block_sum2(s2, 0.f, red[1]).x * inv_h + eps);
    } else {
      r = rsqrtf(tot * inv_h + eps);
    }
    if (threadIdx.x == 0) {
      rstd_ws[row] = r;
      if (LN) mean_ws[row] = mu;
    }
  }
  float s_a = 0.f, s_b = 0.f;
  for (int c = threadIdx.x; c < hidden; c += kThreads) {
    const float xf = Ev<T>::f(xr[c]), dxh = Ev<T>::f(dyr[c]) * gamma[c];
    if (LN) {
      const float xh = (xf - mu) * r;
      s_a += dxh;
      s_b += dxh * xh;
    } else {
      s_a += dxh * xf;
    }
  }
  const float2 s = block_sum2(s_a, s_b, red[2]);
  const float c1 = LN ? s.x * inv_h : 0.f;
  const float c2 = LN ? s.y * inv_h : r * r * r * s.x * inv_h;
  T* dxr = dx + row * lddx;
  for (int c = threadIdx.x; c < hidden; c += kThreads) {
    const float xf = Ev<T>::f(xr[c]), dxh = Ev<T>::f(dyr[c]) * gamma[c];
    dxr[c] = Ev<T>::t(LN ? r * (dxh - c1 - (xf - mu) * r * c2) : r * dxh - xf * c2);
  }
}

// Scalar fallback for dgamma / dbeta: one thread per column, rows in order.
template <typename T, bool LN>
__global__ void norm_bwd_cols_kernel(int rows, int hidden, const T* __restrict__ x, long long ldx,
                                     const T* __restrict__ dy, long long lddy, const float* __restrict__ mean,
                                     const float* __restrict__ rstd, float* dgamma, float* dbeta) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= hidden) return;
  float sg = 0.f, sb = 0.f;
  for (int row = 0; row < rows; ++row) {
    const float xf = Ev<T>::f(x[(long long)row * ldx + c]), df = Ev<T>::f(dy[(long long)row * lddy + c]);
    const float r = rstd[row];
    sg += LN ? df * ((xf - mean[row]) * r) : df * xf * r;
    sb += df;
  }
  if (dgamma) dgamma[c] = sg;
  if (LN && dbeta) dbeta[c] = sb;
}

template <typename T, bool LN>
cudaError_t bwd_dispatch(const NormBwdArgs& a, int num_sms, void* ws, size_t ws_bytes, cudaStream_t s) {
  constexpr int EPV = 16 / sizeof(T);
  const T* x = static_cast<const T*>(a.x);
  const T* dy = static_cast<const T*>(a.dy);
  T* dx = static_cast<T*>(a.dx);
  const bool want_cols = a.dgamma || (LN && a.dbeta);
  const bool vec = a.hidden % EPV == 0 && a.hidden <= 4 * kThreads * EPV &&
                   reinterpret_cast<uintptr_t>(a.x) % 16 == 0 && reinterpret_cast<uintptr_t>(a.dy) % 16 == 0 &&
                   reinterpret_cast<uintptr_t>(a.dx) % 16 == 0 && reinterpret_cast<uintptr_t>(a.gamma) % 16 == 0 &&
                   (a.ldx * (long long)sizeof(T)) % 16 == 0 && (a.lddy * (long long)sizeof(T)) % 16 == 0 &&
                   (a.lddx * (long long)sizeof(T)) % 16 == 0;
  if (vec) {
    const int nv = (a.hidden / EPV + kThreads - 1) / kThreads;
    auto pick = [&](auto kfn) -> cudaError_t {
      int occ = 0;
      cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kfn, kThreads, 0);
      if (e != cudaSuccess) return e;
      if (occ < 1) occ = 1;
      long long g = (long long)num_sms * occ;
      if (g > a.rows) g = a.rows;
      float* part = nullptr;
      if (want_cols) {
        const size_t need = (size_t)g * a.hidden * sizeof(float) * (LN ? 2 : 1);
        if (!ws || ws_bytes < need) return cudaErrorMemoryAllocation;
        part = static_cast<float*>(ws);
      }
      {
        ProfLaunch prof("norm_bwd_vec_kernel", dim3((unsigned)g), dim3(kThreads), 0, s);
        kfn<<<(unsigned)g, kThreads, 0, s>>>(a.rows, a.hidden, x, a.ldx, dy, a.lddy, a.gamma, a.mean, a.rstd, a.eps,
                                             dx, a.lddx, part);
        e = cudaGetLastError();
        if (e != cudaSuccess) return e;
      }
      if (want_cols) {
        const dim3 sg((a.hidden + kSumCols - 1) / kSumCols, LN ? 2 : 1);
        ProfLaunch prof("norm_bwd_sum_parts_kernel", sg, dim3(kSumCols * kSumWarps), 0, s);
        norm_bwd_sum_parts_kernel<<<sg, kSumCols * kSumWarps, 0, s>>>(a.hidden, (int)g, part, a.dgamma,
                                                                      LN ? a.dbeta : nullptr);
        e = cudaGetLastError();
      }
      return e;
    };
    const bool pf = !getenv("GRX_NORM_BWD_NO_PREFETCH");
    if (nv <= 1) return pf ? pick(norm_bwd_vec_kernel<T, 1, LN, true>) : pick(norm_bwd_vec_kernel<T, 1, LN>);
    if (nv <= 2) return pf ? pick(norm_bwd_vec_kernel<T, 2, LN, true>) : pick(norm_bwd_vec_kernel<T, 2, LN>);
    return pf ? pick(norm_bwd_vec_kernel<T, 4, LN, true>) : pick(norm_bwd_vec_kernel<T, 4, LN>);
  }
  // Scalar path: statistics go to scratch when not supplied.
  const float* mean = a.mean;
  const float* rstd = a.rstd;
  float* mean_ws = nullptr;
  float* rstd_ws = nullptr;
  if (!a.rstd) {
    if (!ws || ws_bytes < (size_t)a.rows * 2 * sizeof(float)) return cudaErrorMemoryAllocation;
    rstd_ws = static_cast<float*>(ws);
    mean_ws = rstd_ws + a.rows;
    rstd = rstd_ws;
    mean = mean_ws;
  }
  {
    ProfLaunch prof("norm_bwd_row_scalar_kernel", dim3(a.rows), dim3(kThreads), 0, s);
    norm_bwd_row_scalar_kernel<T, LN><<<a.rows, kThreads, 0, s>>>(a.hidden, x, a.ldx, dy, a.lddy, a.gamma, a.mean,
                                                                  a.rstd, a.eps, dx, a.lddx, mean_ws, rstd_ws);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  if (want_cols) {
    ProfLaunch prof("norm_bwd_cols_kernel", dim3((a.hidden + 255) / 256), dim3(256), 0, s);
    norm_bwd_cols_kernel<T, LN><<<(a.hidden + 255) / 256, 256, 0, s>>>(a.rows, a.hidden, x, a.ldx, dy, a.lddy, mean,
                                                                       rstd, a.dgamma, LN ? a.dbeta : nullptr);
    return cudaGetLastError();
  }
  return cudaSuccess;
}

}  // namespace

size_t norm_bwd_workspace_bytes(int rows, int hidden, bool layernorm, int num_sms) {
  // Upper bound over both paths: G <= num_sms * 8 resident 256-thread CTAs.
  const size_t g = (size_t)num_sms * 8 < (size_t)rows ? (size_t)num_sms * 8 : (size_t)rows;
  const size_t parts = g * (size_t)hidden * sizeof(float) * (layernorm ? 2 : 1);
  const size_t stats = (size_t)rows * 2 * sizeof(float);
  return parts > stats ? parts : stats;
}

cudaError_t launch_norm_bwd(const NormBwdArgs& a, int num_sms, void* ws, size_t ws_bytes, cudaStream_t s) {
  switch (a.dtype * 2 + (a.layernorm ? 1 : 0)) {
    case 0: return bwd_dispatch<float, false>(a, num_sms, ws, ws_bytes, s);
    case 1: return bwd_dispatch<float, true>(a, num_sms, ws, ws_bytes, s);
    case 2: return bwd_dispatch<__nv_bfloat16, false>(a, num_sms, ws, ws_bytes, s);
    case 3: return bwd_dispatch<__nv_bfloat16, true>(a, num_sms, ws, ws_bytes, s);
    case 4: return bwd_dispatch<__half, false>(a, num_sms, ws, ws_bytes, s);
    case 5: return bwd_dispatch<__half, true>(a, num_sms, ws, ws_bytes, s);
  }
  return cudaErrorInvalidValue;
}

}  // namespace grx
