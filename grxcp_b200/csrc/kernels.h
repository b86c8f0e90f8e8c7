// Host-callable launchers of the non-tcgen05 kernels. Each enqueues on the
// given stream and returns the launch status; none synchronises.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "grx/grx_cycles.h"

namespace grx {

struct SgemmArgs {
  int m, n, k, batch;
  int ta, tb;
  float alpha, beta;
  const float* a; long long lda, stride_a;
  const float* b; long long ldb, stride_b;
  float* c; long long ldc, stride_c;
  grxCycleSlot* probe;  // one slot per CTA, or null
};
cudaError_t launch_sgemm(const SgemmArgs& a, int num_sms, cudaStream_t s);
// CTAs the sgemm kernel launches for an m x n x batch problem on num_sms SMs
// (one probe slot each).
int sgemm_ctas(int m, int n, int batch, int num_sms);

// Copies op(X) (R rows of the MN extent by K) into a dense K-major buffer
// dst[b][r][kk] with row pitch ldp elements. es = element bytes (1 or 2).
cudaError_t launch_pack_kmajor(const void* src, int es, int src_mn_major, long long ld, long long stride, int batch,
                               int rows, int k, void* dst, long long ldp, cudaStream_t s);

// The k == 0 GEMM: C = act(beta*C (+ bias[j] or bias[i])) over the m x n window of every batch
// member; out: 0 f32, 1 bf16, 2 f16, 3 s32 (integer beta).
cudaError_t launch_gemm_k0(int out, void* c, long long ldc, long long stride_c, int m, int n, int batch,
                           float beta, int ibeta, const void* bias, int bias_bf16, long long stride_bias,
                           int bias_rows, int act, cudaStream_t s);

cudaError_t launch_saxpy(int n, float alpha, const float* x, int incx, float* y, int incy, cudaStream_t s);
cudaError_t launch_sscal(int n, float alpha, float* x, int incx, cudaStream_t s);
cudaError_t launch_sgemv(int trans, int m, int n, float alpha, const float* a, int lda, const float* x, int incx,
                         float beta, float* y, int incy, cudaStream_t s);

// Norms (norm.cu). dtype: 0 f32, 1 bf16, 2 f16 (x and y alike).
cudaError_t launch_rmsnorm(int rows, int hidden, int dtype, const void* x, long long ldx, const float* gamma,
                           float eps, void* y, long long ldy, float* rstd, cudaStream_t s);
cudaError_t launch_layernorm(int rows, int hidden, int dtype, const void* x, long long ldx, const float* gamma,
                             const float* beta, float eps, void* y, long long ldy, float* mean, float* rstd,
                             cudaStream_t s);

// Softmax over each row / element-wise activation (softmax.cu); dtype as norms,
// act a grx::kAct* value.
// conv2d direct fallback and pooling (conv.cu), NHWC activations, KRSC
// filters. dtype codes: 0 f32, 1 bf16, 2 f16.
struct ConvArgs {
  int n, h, w, c, k, r, s, p, q;
  int pad_h, pad_w, stride_h, stride_w, dil_h, dil_w;
  int in_dtype, out_dtype;
  const void* x;
  const void* filt;
  void* y;
  const float* bias;
  float alpha, beta;
  int act;
};
cudaError_t launch_conv2d_direct(const ConvArgs& a, int num_sms, cudaStream_t s);
struct PoolArgs {
  int n, h, w, c, r, s, p, q;
  int pad_h, pad_w, stride_h, stride_w;
  int mode;  // 0 max, 1 average over r*s, 2 average over in-image taps
  int dtype;
  const void* x;
  void* y;
};
cudaError_t launch_pool2d(const PoolArgs& a, int num_sms, cudaStream_t s);

// RMSNorm / LayerNorm backward (norm_bwd.cu). mean/rstd: saved statistics
// or null (recomputed); dgamma/dbeta may be null. ws: scratch of at least
// norm_bwd_workspace_bytes when dgamma/dbeta are wanted or stats are null.
struct NormBwdArgs {
  int rows, hidden, dtype;  // dtype 0 f32, 1 bf16, 2 f16
  bool layernorm;
  const void* x; long long ldx;
  const void* dy; long long lddy;
  const float* gamma;
  const float* mean;
  const float* rstd;
  float eps;
  void* dx; long long lddx;
  float* dgamma;
  float* dbeta;
};
size_t norm_bwd_workspace_bytes(int rows, int hidden, bool layernorm, int num_sms);
cudaError_t launch_norm_bwd(const NormBwdArgs& a, int num_sms, void* ws, size_t ws_bytes, cudaStream_t s);

cudaError_t launch_softmax(int rows, int cols, int dtype, const void* x, long long ldx, void* y, long long ldy,
                           cudaStream_t s);
cudaError_t launch_gelu(long long n, int dtype, const void* x, void* y, int act, int num_sms, cudaStream_t s);
cudaError_t launch_softmax_bwd(int rows, int cols, int dtype, const void* y, long long ldy, const void* dy,
                               long long lddy, void* dx, long long lddx, cudaStream_t s);
cudaError_t launch_gelu_bwd(long long n, int dtype, const void* x, const void* dy, void* dx, int act, int num_sms,
                            cudaStream_t s);

// Test hook: one CTA waits on an mbarrier nothing ever arrives at, through the
// same bounded wait every kernel uses, and must come back with kErrTimeoutTest
// in *err_word after about timeout_ns.
cudaError_t launch_bounded_wait_probe(int* err_word, unsigned long long timeout_ns, cudaStream_t s);

}  // namespace grx
