// FP32-pipe and memory-bound grxBLAS kernels for sm_100a: SGEMM (exact fp32
// FFMA, no TF32), the operand packer and k == 0 epilogue of the tensor-core
// path, and level-1/2 BLAS.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "activation.cuh"
#include "kernels.h"
#include "profile.h"
#include "ptx.cuh"

namespace grx {

// ---------------------------------------------------------------- SGEMM
//
// Same contract as the reference sgemm kernel (src/libs/grxblas/kernels/
// sgemm.cpp:22-89): column-major, op(A)(i,l) = ta ? A[l + i*lda] : A[i + l*lda],
// op(B)(l,j) = tb ? B[j + l*ldb] : B[l + j*ldb], batch on the grid, signed
// element strides, beta == 0 never reads C. Instead of one thread per output
// with two global loads per multiply-add, a 128 x 128 output tile per CTA is
// staged through shared memory in k-slabs of 8 and each thread accumulates an
// 8 x 8 sub-tile in registers (fp32 FMA, one accumulator per output, k in
// ascending order).
constexpr int SG_BM = 128, SG_BN = 128, SG_BK = 8, SG_THREADS = 256;

__global__ void __launch_bounds__(SG_THREADS) sgemm_kernel(SgemmArgs p) {
  __shared__ __align__(16) float As[2][SG_BK][SG_BM];
  __shared__ __align__(16) float Bs[2][SG_BK][SG_BN];
  long long t_start = 0;
  if (p.probe) t_start = clock64();

  const int bz = blockIdx.z;
  const float* A = p.a + (long long)bz * p.stride_a;
  const float* B = p.b + (long long)bz * p.stride_b;
  float* C = p.c + (long long)bz * p.stride_c;
  const int m0 = blockIdx.x * SG_BM, n0 = blockIdx.y * SG_BN;
  const int tid = threadIdx.x;
  const int tx = tid & 15, ty = tid >> 4;

  // Load mapping: 1024 elements per operand slab, 4 per thread. The fastest
  // index follows the operand's contiguous direction.
  auto load_slab = [&](int buf, int k0) {
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int idx = tid + e * SG_THREADS;
      int r, l;  // A: r in [0,128) rows of op(A), l in [0,8)
      if (!p.ta) { r = idx & 127; l = idx >> 7; } else { l = idx & 7; r = idx >> 3; }
      const int gi = m0 + r, gl = k0 + l;
      float v = 0.f;
      if (gi < p.m && gl < p.k) v = p.ta ? A[gl + (long long)gi * p.lda] : A[gi + (long long)gl * p.lda];
      As[buf][l][r] = v;
      int c, lb;  // B: c in [0,128) columns of op(B)
      if (!p.tb) { lb = idx & 7; c = idx >> 3; } else { c = idx & 127; lb = idx >> 7; }
      const int gj = n0 + c, gl2 = k0 + lb;
      float w = 0.f;
      if (gj < p.n && gl2 < p.k) w = p.tb ? B[gj + (long long)gl2 * p.ldb] : B[gl2 + (long long)gj * p.ldb];
      Bs[buf][lb][c] = w;
    }
  };

  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;

  const int kt = (p.k + SG_BK - 1) / SG_BK;
  if (kt > 0) load_slab(0, 0);
  __syncthreads();
  for (int t = 0; t < kt; ++t) {
    const int cur = t & 1;
    if (t + 1 < kt) load_slab(cur ^ 1, (t + 1) * SG_BK);
#pragma unroll
    for (int l = 0; l < SG_BK; ++l) {
      float a[8], b[8];
      const float4 a0 = *reinterpret_cast<const float4*>(&As[cur][l][tx * 4]);
      const float4 a1 = *reinterpret_cast<const float4*>(&As[cur][l][64 + tx * 4]);
      const float4 b0 = *reinterpret_cast<const float4*>(&Bs[cur][l][ty * 4]);
      const float4 b1 = *reinterpret_cast<const float4*>(&Bs[cur][l][64 + ty * 4]);
      a[0] = a0.x; a[1] = a0.y; a[2] = a0.z; a[3] = a0.w; a[4] = a1.x; a[5] = a1.y; a[6] = a1.z; a[7] = a1.w;
      b[0] = b0.x; b[1] = b0.y; b[2] = b0.z; b[3] = b0.w; b[4] = b1.x; b[5] = b1.y; b[6] = b1.z; b[7] = b1.w;
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }

#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int gj = n0 + (j < 4 ? ty * 4 + j : 64 + ty * 4 + (j - 4));
    if (gj >= p.n) continue;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int gi = m0 + (i < 4 ? tx * 4 + i : 64 + tx * 4 + (i - 4));
      if (gi >= p.m) continue;
      const long long ci = gi + (long long)gj * p.ldc;
      const float v = __fmul_rn(p.alpha, acc[i][j]);
      C[ci] = (p.beta == 0.f) ? v : __fadd_rn(v, __fmul_rn(p.beta, C[ci]));
    }
  }

  if (p.probe && tid == 0) {
    const unsigned lin = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);
    unsigned smid;
    asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
    grxCycleSlot s;
    s.start = (uint64_t)t_start;
    s.end = (uint64_t)clock64();
    s.core = smid;
    s.warp = lin;
    p.probe[lin] = s;
  }
}

int sgemm_ctas(int m, int n) {
  if (m <= 0 || n <= 0) return 0;
  return ((m + SG_BM - 1) / SG_BM) * ((n + SG_BN - 1) / SG_BN);
}

cudaError_t launch_sgemm(const SgemmArgs& a, cudaStream_t s) {
  dim3 grid((a.m + SG_BM - 1) / SG_BM, (a.n + SG_BN - 1) / SG_BN, a.batch);
  if (grid.y > 65535u || grid.z > 65535u) return cudaErrorInvalidValue;
  ProfLaunch prof("sgemm_kernel", grid, dim3(SG_THREADS), 0, s);
  sgemm_kernel<<<grid, SG_THREADS, 0, s>>>(a);
  return cudaGetLastError();
}

// ---------------------------------------------------------------- packing

template <typename T>
__global__ void pack_kmajor_kernel(const T* __restrict__ src, int mn_major, long long ld, long long stride,
                                   int rows, int k, T* __restrict__ dst, long long ldp, long long total) {
  for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total;
       e += (long long)gridDim.x * blockDim.x) {
    const long long per = (long long)rows * ldp;
    const long long b = e / per;
    const long long rem = e - b * per;
    const long long r = rem / ldp;
    const long long kk = rem - r * ldp;
    T v{};
    if (kk < k) {
      const T* s = src + b * stride;
      v = mn_major ? s[r + kk * ld] : s[kk + r * ld];
    }
    dst[e] = v;
  }
}

cudaError_t launch_pack_kmajor(const void* src, int es, int src_mn_major, long long ld, long long stride, int batch,
                               int rows, int k, void* dst, long long ldp, cudaStream_t s) {
  const long long total = (long long)batch * rows * ldp;
  if (total == 0) return cudaSuccess;
  const int threads = 256;
  long long blocks = (total + threads - 1) / threads;
  if (blocks > 148LL * 64) blocks = 148LL * 64;
  ProfLaunch prof("pack_kmajor_kernel", dim3((unsigned)blocks), dim3(threads), 0, s);
  if (es == 2)
    pack_kmajor_kernel<uint16_t><<<(unsigned)blocks, threads, 0, s>>>(
        static_cast<const uint16_t*>(src), src_mn_major, ld, stride, rows, k, static_cast<uint16_t*>(dst), ldp,
        total);
  else
    pack_kmajor_kernel<uint8_t><<<(unsigned)blocks, threads, 0, s>>>(static_cast<const uint8_t*>(src),
                                                                      src_mn_major, ld, stride, rows, k,
                                                                      static_cast<uint8_t*>(dst), ldp, total);
  return cudaGetLastError();
}

// ---------------------------------------------------------------- k == 0

template <int OUT>
__global__ void gemm_k0_kernel(void* c, long long ldc, long long stride_c, int m, int n, float beta, int ibeta,
                               const void* bias, int bias_bf16, long long stride_bias, int bias_rows, int act) {
  const int b = blockIdx.z;
  const int j = blockIdx.y;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < m; i += gridDim.x * blockDim.x) {
    const long long idx = (long long)b * stride_c + i + (long long)j * ldc;
    if constexpr (OUT == 3) {
      int* C = static_cast<int*>(c);
      C[idx] = ibeta == 0 ? 0 : ibeta * C[idx];
    } else {
      float v = 0.f;
      if (beta != 0.f) {
        float cv;
        if constexpr (OUT == 0) cv = static_cast<float*>(c)[idx];
        else if constexpr (OUT == 1) cv = __bfloat162float(static_cast<__nv_bfloat16*>(c)[idx]);
        else cv = __half2float(static_cast<__half*>(c)[idx]);
        v = __fmul_rn(beta, cv);
      }
      if (bias) {
        const long long bi = (long long)b * stride_bias + (bias_rows ? i : j);
        v = __fadd_rn(v, bias_bf16 ? __bfloat162float(static_cast<const __nv_bfloat16*>(bias)[bi])
                                   : static_cast<const float*>(bias)[bi]);
      }
      v = apply_act(v, act);
      if constexpr (OUT == 0) static_cast<float*>(c)[idx] = v;
      else if constexpr (OUT == 1) static_cast<__nv_bfloat16*>(c)[idx] = __float2bfloat16_rn(v);
      else static_cast<__half*>(c)[idx] = __float2half_rn(v);
    }
  }
}

cudaError_t launch_gemm_k0(int out, void* c, long long ldc, long long stride_c, int m, int n, int batch,
                           float beta, int ibeta, const void* bias, int bias_bf16, long long stride_bias,
                           int bias_rows, int act, cudaStream_t s) {
  if (n > 65535 || batch > 65535) return cudaErrorInvalidValue;
  dim3 grid((m + 255) / 256, n, batch);
  ProfLaunch prof("gemm_k0_kernel", grid, dim3(256), 0, s);
  switch (out) {
    case 0: gemm_k0_kernel<0><<<grid, 256, 0, s>>>(c, ldc, stride_c, m, n, beta, ibeta, bias, bias_bf16, stride_bias, bias_rows, act); break;
    case 1: gemm_k0_kernel<1><<<grid, 256, 0, s>>>(c, ldc, stride_c, m, n, beta, ibeta, bias, bias_bf16, stride_bias, bias_rows, act); break;
    case 2: gemm_k0_kernel<2><<<grid, 256, 0, s>>>(c, ldc, stride_c, m, n, beta, ibeta, bias, bias_bf16, stride_bias, bias_rows, act); break;
    case 3: gemm_k0_kernel<3><<<grid, 256, 0, s>>>(c, ldc, stride_c, m, n, beta, ibeta, bias, bias_bf16, stride_bias, bias_rows, act); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

// ---------------------------------------------------------------- level 1/2
//
// Vector element i of a length-n vector with increment inc sits at
// inc > 0 ? i*inc : (n-1-i)*(-inc) (reference grxblas.h:160-166,
// kernels/blas12.cpp:33).
__device__ __forceinline__ long long vec_at(long long i, long long n, int inc) {
  return inc > 0 ? i * inc : (n - 1 - i) * (long long)(-inc);
}

__global__ void saxpy_kernel(int n, float alpha, const float* x, int incx, float* y, int incy) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    float* yp = y + vec_at(i, n, incy);
    *yp = fmaf(alpha, x[vec_at(i, n, incx)], *yp);
  }
}

__global__ void sscal_kernel(int n, float alpha, float* x, int incx) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
    x[i * incx] = alpha * x[i * incx];
}

// y = alpha*A*x + beta*y, one thread per output row (column-major A: a warp's
// loads of one column are contiguous).
__global__ void sgemv_n_kernel(int m, int n, float alpha, const float* a, int lda, const float* x, int incx,
                               float beta, float* y, int incy) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= m) return;
  float acc = 0.f;
  for (int j = 0; j < n; ++j) acc = fmaf(a[i + (long long)j * lda], x[vec_at(j, n, incx)], acc);
  float* yp = y + vec_at(i, m, incy);
  *yp = beta == 0.f ? alpha * acc : fmaf(alpha, acc, beta * *yp);
}

// y = alpha*A^T*x + beta*y, one warp per output (lanes walk down a column).
__global__ void sgemv_t_kernel(int m, int n, float alpha, const float* a, int lda, const float* x, int incx,
                               float beta, float* y, int incy) {
  const int j = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (j >= n) return;
  float acc = 0.f;
  for (int i = lane; i < m; i += 32) acc = fmaf(a[i + (long long)j * lda], x[vec_at(i, m, incx)], acc);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (lane == 0) {
    float* yp = y + vec_at(j, n, incy);
    *yp = beta == 0.f ? alpha * acc : fmaf(alpha, acc, beta * *yp);
  }
}

static unsigned grid_for(long long n, int threads) {
  long long b = (n + threads - 1) / threads;
  if (b > 148LL * 32) b = 148LL * 32;
  return (unsigned)(b < 1 ? 1 : b);
}

cudaError_t launch_saxpy(int n, float alpha, const float* x, int incx, float* y, int incy, cudaStream_t s) {
  ProfLaunch prof("saxpy_kernel", dim3(grid_for(n, 256)), dim3(256), 0, s);
  saxpy_kernel<<<grid_for(n, 256), 256, 0, s>>>(n, alpha, x, incx, y, incy);
  return cudaGetLastError();
}

cudaError_t launch_sscal(int n, float alpha, float* x, int incx, cudaStream_t s) {
  ProfLaunch prof("sscal_kernel", dim3(grid_for(n, 256)), dim3(256), 0, s);
  sscal_kernel<<<grid_for(n, 256), 256, 0, s>>>(n, alpha, x, incx);
  return cudaGetLastError();
}

cudaError_t launch_sgemv(int trans, int m, int n, float alpha, const float* a, int lda, const float* x, int incx,
                         float beta, float* y, int incy, cudaStream_t s) {
  ProfLaunch prof(trans ? "sgemv_t_kernel" : "sgemv_n_kernel", dim3(trans ? (n + 3) / 4 : (m + 127) / 128), dim3(128), 0, s);
  if (!trans)
    sgemv_n_kernel<<<(m + 127) / 128, 128, 0, s>>>(m, n, alpha, a, lda, x, incx, beta, y, incy);
  else
    sgemv_t_kernel<<<(n + 3) / 4, 128, 0, s>>>(m, n, alpha, a, lda, x, incx, beta, y, incy);
  return cudaGetLastError();
}

// ---------------------------------------------------------------- wait probe

__global__ void bounded_wait_probe_kernel(int* err_word, unsigned long long timeout_ns) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    WaitCtx wc{err_word, &abort_flag, timeout_ns};
    wait_bounded(&bar, 0, wc, kErrTimeoutTest);  // nothing ever arrives
  }
  __syncthreads();
}

cudaError_t launch_bounded_wait_probe(int* err_word, unsigned long long timeout_ns, cudaStream_t s) {
  bounded_wait_probe_kernel<<<1, 32, 0, s>>>(err_word, timeout_ns);
  return cudaGetLastError();
}

}  // namespace grx
