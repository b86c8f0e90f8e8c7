// Runs the reference's sgemm kernel (compiled for the host from its own source,
// src/libs/grxblas/kernels/sgemm.cpp) over a grid, serially, exactly as the
// reference host library launches it (src/libs/grxblas/grxblas.cpp:904-938:
// block = warp, grid = (ceil(m*n / warp), batch)). TEST INFRASTRUCTURE ONLY.
#include <stddef.h>

#include <grx/device/grx_cycles.h>

#include "sgemm_abi.h"

thread_local grx_ref_dim3 blockIdx, blockDim, threadIdx, gridDim;

void sgemm(grxblas_sgemm_args* arg);

extern "C" void ref_sgemm_run(int ta, int tb, int m, int n, int k, float alpha, const float* A, int lda,
                              long long sA, const float* B, int ldb, long long sB, float beta, float* C, int ldc,
                              long long sC, int batch) {
  grxblas_sgemm_args a{};
  a.abi_version = GRXBLAS_SGEMM_ABI_VERSION;
  a.m = (uint32_t)m; a.n = (uint32_t)n; a.k = (uint32_t)k;
  a.lda = (uint32_t)lda; a.ldb = (uint32_t)ldb; a.ldc = (uint32_t)ldc;
  a.transa = (uint32_t)ta; a.transb = (uint32_t)tb;
  a.alpha = alpha; a.beta = beta;
  a.a = (uint64_t)(uintptr_t)A; a.b = (uint64_t)(uintptr_t)B; a.c = (uint64_t)(uintptr_t)C;
  a.batch = (uint32_t)batch;
  a.stride_a = sA; a.stride_b = sB; a.stride_c = sC;
  const uint32_t warp = 32;
  const uint32_t total = (uint32_t)((size_t)m * (size_t)n);
  const uint32_t grid = (total + warp - 1) / warp;
  blockDim = {warp, 1, 1};
  gridDim = {grid, (uint32_t)batch, 1};
  for (uint32_t by = 0; by < (uint32_t)batch; ++by)
    for (uint32_t bx = 0; bx < grid; ++bx)
      for (uint32_t t = 0; t < warp; ++t) {
        blockIdx = {bx, by, 0};
        threadIdx = {t, 0, 0};
        sgemm(&a);
      }
}
