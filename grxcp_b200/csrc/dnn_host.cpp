// grxDNN host library for B200: handle, validation, dispatch.
//
// The reference has no grxDNN code (planned only: docs/designs/
// grxcp_architecture.md:594, docs/designs/grxcp_roadmap.md:860-876), so the
// validation rules here are this library's own, written in grxBLAS's style
// (reference src/libs/grxblas/grxblas.cpp:498-524): null handle ->
// NOT_INITIALIZED, malformed arguments -> INVALID_VALUE, empty problem ->
// SUCCESS without a launch, a type or shape the kernels do not implement ->
// NOT_SUPPORTED (never a slower substitute).
#include <cuda_runtime.h>

#include <math.h>

#include <mutex>

#include "attention.cuh"
#include "gemm_tc.cuh"
#include "grx/grxdnn.h"
#include "host_common.h"
#include "kernels.h"

struct grxdnnContext {
  cudaStream_t stream = nullptr;
  std::mutex mutex;
  grx::DeviceState dev;
  void* ws = nullptr;  // grow-only, stream-ordered scratch (norm backward)
  size_t ws_bytes = 0;
};

namespace {

grxdnnStatus_t from_cuda(cudaError_t e) {
  switch (e) {
    case cudaSuccess: return GRXDNN_STATUS_SUCCESS;
    case cudaErrorMemoryAllocation: return GRXDNN_STATUS_ALLOC_FAILED;
    case cudaErrorInvalidValue: return GRXDNN_STATUS_INVALID_VALUE;
    case cudaErrorNotSupported: return GRXDNN_STATUS_NOT_SUPPORTED;
    case cudaErrorNoKernelImageForDevice:
    case cudaErrorInvalidDeviceFunction: return GRXDNN_STATUS_ARCH_MISMATCH;
    default: return GRXDNN_STATUS_EXECUTION_FAILED;
  }
}

grxdnnStatus_t ensure(grxdnnContext& ctx, bool need_tensor) {
  std::lock_guard<std::mutex> lock(ctx.mutex);
  const int rc = grx::ensure_device(ctx.dev);
  if (rc == 1) return GRXDNN_STATUS_NOT_INITIALIZED;
  if (rc == 2) return GRXDNN_STATUS_ALLOC_FAILED;
  if (need_tensor && ctx.dev.cc_major != 10) return GRXDNN_STATUS_ARCH_MISMATCH;
  return GRXDNN_STATUS_SUCCESS;
}

int norm_dtype(grxDataType_t t) {
  switch (t) {
    case GRX_R_32F: return 0;
    case GRX_R_16BF: return 1;
    case GRX_R_16F: return 2;
    default: return -1;
  }
}

grxdnnStatus_t check_norm(grxdnnHandle_t h, int rows, int hidden, const void* x, grxDataType_t xt, long long ldx,
                          const float* gamma, float eps, const void* y, grxDataType_t yt, long long ldy,
                          bool& empty) {
  empty = false;
  if (!h) return GRXDNN_STATUS_NOT_INITIALIZED;
  if (rows < 0 || hidden < 0) return GRXDNN_STATUS_INVALID_VALUE;
  if (rows == 0) {
    empty = true;
    return GRXDNN_STATUS_SUCCESS;
  }
  if (hidden == 0) return GRXDNN_STATUS_INVALID_VALUE;
  if (!x || !y || !gamma) return GRXDNN_STATUS_INVALID_VALUE;
  if (ldx < hidden || ldy < hidden) return GRXDNN_STATUS_INVALID_VALUE;
  if (!(eps >= 0.0f)) return GRXDNN_STATUS_INVALID_VALUE;
  if (xt != yt || norm_dtype(xt) < 0) return GRXDNN_STATUS_NOT_SUPPORTED;
  return GRXDNN_STATUS_SUCCESS;
}

void* workspace(grxdnnContext& ctx, size_t bytes) {
  std::lock_guard<std::mutex> lock(ctx.mutex);
  if (ctx.ws_bytes >= bytes) return ctx.ws;
  if (grx::fault_injected("alloc")) return nullptr;
  if (ctx.ws) cudaFreeAsync(ctx.ws, ctx.stream);
  ctx.ws = nullptr;
  ctx.ws_bytes = 0;
  void* p = nullptr;
  if (cudaMallocAsync(&p, bytes, ctx.stream) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  ctx.ws = p;
  ctx.ws_bytes = bytes;
  return p;
}

grxdnnStatus_t norm_backward(grxdnnHandle_t handle, bool ln, int rows, int hidden, const void* dy,
                             grxDataType_t dyType, long long lddy, const void* x, grxDataType_t xType, long long ldx,
                             const float* gamma, const float* mean, const float* rstd, float eps, void* dx,
                             grxDataType_t dxType, long long lddx, float* dgamma, float* dbeta) {
  bool empty;
  grxdnnStatus_t s = check_norm(handle, rows, hidden, x, xType, ldx, gamma, eps, dx, dxType, lddx, empty);
  if (s != GRXDNN_STATUS_SUCCESS) return s;
  if (!empty) {
    if (!dy || lddy < hidden) return GRXDNN_STATUS_INVALID_VALUE;
    if (ln && ((mean == nullptr) != (rstd == nullptr))) return GRXDNN_STATUS_INVALID_VALUE;
    if (dyType != xType) return GRXDNN_STATUS_NOT_SUPPORTED;
  }
  auto& ctx = *reinterpret_cast<grxdnnContext*>(handle);
  if (empty) {
    // No rows: the parameter gradients are sums over nothing.
    if (!dgamma && !dbeta) return GRXDNN_STATUS_SUCCESS;
    if (hidden <= 0) return hidden < 0 ? GRXDNN_STATUS_INVALID_VALUE : GRXDNN_STATUS_SUCCESS;
    s = ensure(ctx, false);
    if (s != GRXDNN_STATUS_SUCCESS) return s;
    if (dgamma) {
      const cudaError_t e = cudaMemsetAsync(dgamma, 0, (size_t)hidden * sizeof(float), ctx.stream);
      if (e != cudaSuccess) return from_cuda(e);
    }
    if (ln && dbeta) return from_cuda(cudaMemsetAsync(dbeta, 0, (size_t)hidden * sizeof(float), ctx.stream));
    return GRXDNN_STATUS_SUCCESS;
  }
  s = ensure(ctx, false);
  if (s != GRXDNN_STATUS_SUCCESS) return s;
  const bool need_ws = dgamma || (ln && dbeta) || !rstd;
  void* ws = nullptr;
  size_t ws_bytes = 0;
  if (need_ws) {
    ws_bytes = grx::norm_bwd_workspace_bytes(rows, hidden, ln, ctx.dev.num_sms);
    ws = workspace(ctx, ws_bytes);
    if (!ws) return GRXDNN_STATUS_ALLOC_FAILED;
  }
  grx::NormBwdArgs a{};
  a.rows = rows;
  a.hidden = hidden;
  a.dtype = norm_dtype(xType);
  a.layernorm = ln;
  a.x = x; a.ldx = ldx;
  a.dy = dy; a.lddy = lddy;
  a.gamma = gamma;
  a.mean = ln ? mean : nullptr;
  a.rstd = rstd;
  a.eps = eps;
  a.dx = dx; a.lddx = lddx;
  a.dgamma = dgamma;
  a.dbeta = ln ? dbeta : nullptr;
  return from_cuda(grx::launch_norm_bwd(a, ctx.dev.num_sms, ws, ws_bytes, ctx.stream));
}

bool same_shape(const grxdnnAttnTensor_t& a, const grxdnnAttnTensor_t& b) {
  return a.batch == b.batch && a.heads == b.heads && a.seq == b.seq && a.headDim == b.headDim;
}

}  // namespace

extern "C" {

const char* grxdnnGetStatusString(grxdnnStatus_t s) {
  switch (s) {
    case GRXDNN_STATUS_SUCCESS: return "success";
    case GRXDNN_STATUS_NOT_INITIALIZED: return "library not initialized (no usable device)";
    case GRXDNN_STATUS_ALLOC_FAILED: return "allocation failed";
    case GRXDNN_STATUS_INVALID_VALUE: return "invalid argument";
    case GRXDNN_STATUS_ARCH_MISMATCH: return "device lacks a required capability (sm_100 tensor cores)";
    case GRXDNN_STATUS_EXECUTION_FAILED: return "kernel execution failed";
    case GRXDNN_STATUS_NOT_SUPPORTED: return "not supported";
    case GRXDNN_STATUS_INTERNAL_ERROR: return "internal error";
  }
  return "unknown status";
}

grxdnnStatus_t grxdnnCreate(grxdnnHandle_t* handle) {
  if (!handle) return GRXDNN_STATUS_INVALID_VALUE;
  *handle = reinterpret_cast<grxdnnHandle_t>(new grxdnnContext());
  return GRXDNN_STATUS_SUCCESS;
}

grxdnnStatus_t grxdnnDestroy(grxdnnHandle_t handle) {
  if (!handle) return GRXDNN_STATUS_NOT_INITIALIZED;
  auto* ctx = reinterpret_cast<grxdnnContext*>(handle);
  if (ctx->ws) {
    cudaFreeAsync(ctx->ws, ctx->stream);
    cudaStreamSynchronize(ctx->stream);
  }
  grx::release_device(ctx->dev);
  delete ctx;
  return GRXDNN_STATUS_SUCCESS;
}

grxdnnStatus_t grxdnnSetStream(grxdnnHandle_t handle, grxStream_t stream) {
  if (!handle) return GRXDNN_STATUS_NOT_INITIALIZED;
  auto* ctx = reinterpret_cast<grxdnnContext*>(handle);
  std::lock_guard<std::mutex> lock(ctx->mutex);
  ctx->stream = reinterpret_cast<cudaStream_t>(stream);
  return GRXDNN_STATUS_SUCCESS;
}

grxdnnStatus_t grxdnnGetStream(grxdnnHandle_t handle, grxStream_t* stream) {
  if (!handle || !stream) return GRXDNN_STATUS_INVALID_VALUE;
  *stream = reinterpret_cast<grxStream_t>(reinterpret_cast<grxdnnContext*>(handle)->stream);
  return GRXDNN_STATUS_SUCCESS;
}

grxdnnStatus_t grxdnnRMSNormForward(grxdnnHandle_t handle, int rows, int hidden, const void* x,
                                    grxDataType_t xType, long long ldx, const float* gamma, float eps, void* y,
                                    grxDataType_t yType, long long ldy, float* rstd) {
  bool empty;
  grxdnnStatus_t s = check_norm(handle, rows, hidden, x, xType, ldx, gamma, eps, y, yType, ldy, empty);
  if (s != GRXDNN_STATUS_SUCCESS || empty) return s;
  auto& ctx = *reinterpret_cast<grxdnnContext*>(handle);
  s = ensure(ctx, false);
  if (s != GRXDNN_STATUS_SUCCESS) return s;
  return from_cuda(
      grx::launch_rmsnorm(rows, hidden, norm_dtype(xType), x, ldx, gamma, eps, y, ldy, rstd, ctx.stream));
}

grxdnnStatus_t grxdnnLayerNormForward(grxdnnHandle_t handle, int rows, int hidden, const void* x,
                                      grxDataType_t xType, long long ldx, const float* gamma, const float* beta,
                                      float eps, void* y, grxDataType_t yType, long long ldy, float* mean,
                                      float* rstd) {
  bool empty;
  grxdnnStatus_t s = check_norm(handle, rows, hidden, x, xType, ldx, gamma, eps, y, yType, ldy, empty);
  if (s != GRXDNN_STATUS_SUCCESS || empty) return s;
  auto& ctx = *reinterpret_cast<grxdnnContext*>(handle);
  s = ensure(ctx, false);
  if (s != GRXDNN_STATUS_SUCCESS) return s;
  return from_cuda(grx::launch_layernorm(rows, hidden, norm_dtype(xType), x, ldx, gamma, beta, eps, y, ldy, mean,
                                         rstd, ctx.stream));
}

grxdnnStatus_t grxdnnRMSNormBackward(grxdnnHandle_t handle, int rows, int hidden, const void* dy,
                                     grxDataType_t dyType, long long lddy, const void* x, grxDataType_t xType,
                                     long long ldx, const float* gamma, const float* rstd, float eps, void* dx,
                                     grxDataType_t dxType, long long lddx, float* dgamma) {
  return norm_backward(handle, false, rows, hidden, dy, dyType, lddy, x, xType, ldx, gamma, nullptr, rstd, eps, dx,
                       dxType, lddx, dgamma, nullptr);
}

grxdnnStatus_t grxdnnLayerNormBackward(grxdnnHandle_t handle, int rows, int hidden, const void* dy,
                                       grxDataType_t dyType, long long lddy, const void* x, grxDataType_t xType,
                                       long long ldx, const float* gamma, const float* mean, const float* rstd,
                                       float eps, void* dx, grxDataType_t dxType, long long lddx, float* dgamma,
                                       float* dbeta) {
  return norm_backward(handle, true, rows, hidden, dy, dyType, lddy, x, xType, ldx, gamma, mean, rstd, eps, dx,
                       dxType, lddx, dgamma, dbeta);
}

grxdnnStatus_t grxdnnSoftmaxForward(grxdnnHandle_t handle, int rows, int cols, const void* x, grxDataType_t xType,
                                    long long ldx, void* y, grxDataType_t yType, long long ldy) {
  if (!handle) return GRXDNN_STATUS_NOT_INITIALIZED;
  if (rows < 0 || cols < 0) return GRXDNN_STATUS_INVALID_VALUE;
  if (rows == 0) return GRXDNN_STATUS_SUCCESS;
  if (cols == 0 || !x || !y || ldx < cols || ldy < cols) return GRXDNN_STATUS_INVALID_VALUE;
  if (xType != yType || norm_dtype(xType) < 0) return GRXDNN_STATUS_NOT_SUPPORTED;
  auto& ctx = *reinterpret_cast<grxdnnContext*>(handle);
  const grxdnnStatus_t s = ensure(ctx, false);
  if (s != GRXDNN_STATUS_SUCCESS) return s;
  return from_cuda(grx::launch_softmax(rows, cols, norm_dtype(xType), x, ldx, y, ldy, ctx.stream));
}

grxdnnStatus_t grxdnnSoftmaxBackward(grxdnnHandle_t handle, int rows, int cols, const void* y, grxDataType_t yType,
                                     long long ldy, const void* dy, grxDataType_t dyType, long long lddy, void* dx,
                                     grxDataType_t dxType, long long lddx) {
  if (!handle) return GRXDNN_STATUS_NOT_INITIALIZED;
  if (rows < 0 || cols < 0) return GRXDNN_STATUS_INVALID_VALUE;
  if (rows == 0) return GRXDNN_STATUS_SUCCESS;
  if (cols == 0 || !y || !dy || !dx || ldy < cols || lddy < cols || lddx < cols) return GRXDNN_STATUS_INVALID_VALUE;
  if (yType != dyType || yType != dxType || norm_dtype(yType) < 0) return GRXDNN_STATUS_NOT_SUPPORTED;
  auto& ctx = *reinterpret_cast<grxdnnContext*>(handle);
  const grxdnnStatus_t s = ensure(ctx, false);
  if (s != GRXDNN_STATUS_SUCCESS) return s;
  return from_cuda(grx::launch_softmax_bwd(rows, cols, norm_dtype(yType), y, ldy, dy, lddy, dx, lddx, ctx.stream));
}

grxdnnStatus_t grxdnnGeluBackward(grxdnnHandle_t handle, long long n, const void* x, const void* dy, void* dx,
                                  grxDataType_t type, grxdnnGeluMode_t mode) {
  if (!handle) return GRXDNN_STATUS_NOT_INITIALIZED;
  if (n < 0 || (unsigned)mode > 1u) return GRXDNN_STATUS_INVALID_VALUE;
  if (n == 0) return GRXDNN_STATUS_SUCCESS;
  if (!x || !dy || !dx) return GRXDNN_STATUS_INVALID_VALUE;
  if (norm_dtype(type) < 0) return GRXDNN_STATUS_NOT_SUPPORTED;
  auto& ctx = *reinterpret_cast<grxdnnContext*>(handle);
  const grxdnnStatus_t s = ensure(ctx, false);
  if (s != GRXDNN_STATUS_SUCCESS) return s;
  const int act = mode == GRXDNN_GELU_ERF ? 3 /*kActGeluErf*/ : 2 /*kActGeluTanh*/;
  return from_cuda(grx::launch_gelu_bwd(n, norm_dtype(type), x, dy, dx, act, ctx.dev.num_sms, ctx.stream));
}

grxdnnStatus_t grxdnnGeluForward(grxdnnHandle_t handle, long long n, const void* x, grxDataType_t xType, void* y,
                                 grxDataType_t yType, grxdnnGeluMode_t mode) {
  if (!handle) return GRXDNN_STATUS_NOT_INITIALIZED;
  if (n < 0 || (unsigned)mode > 1u) return GRXDNN_STATUS_INVALID_VALUE;
  if (n == 0) return GRXDNN_STATUS_SUCCESS;
  if (!x || !y) return GRXDNN_STATUS_INVALID_VALUE;
  if (xType != yType || norm_dtype(xType) < 0) return GRXDNN_STATUS_NOT_SUPPORTED;
  auto& ctx = *reinterpret_cast<grxdnnContext*>(handle);
  const grxdnnStatus_t s = ensure(ctx, false);
  if (s != GRXDNN_STATUS_SUCCESS) return s;
  const int act = mode == GRXDNN_GELU_ERF ? 3 /*kActGeluErf*/ : 2 /*kActGeluTanh*/;
  return from_cuda(grx::launch_gelu(n, norm_dtype(xType), x, y, act, ctx.dev.num_sms, ctx.stream));
}

grxdnnStatus_t grxdnnAttentionForward(grxdnnHandle_t handle, const grxdnnAttnTensor_t* qd, const void* q,
                                      const grxdnnAttnTensor_t* kd, const void* k, const grxdnnAttnTensor_t* vd,
                                      const void* v, const grxdnnAttnTensor_t* od, void* o, float scale, int causal,
                                      float* lse) {
  if (!handle) return GRXDNN_STATUS_NOT_INITIALIZED;
  if (!qd || !kd || !vd || !od) return GRXDNN_STATUS_INVALID_VALUE;
  const grxdnnAttnTensor_t* all[4] = {qd, kd, vd, od};
  for (auto* d : all)
    if (d->batch < 0 || d->heads < 0 || d->seq < 0 || d->headDim <= 0 || d->strideSeq < d->headDim)
      return GRXDNN_STATUS_INVALID_VALUE;
  if (!same_shape(*qd, *od) || !same_shape(*kd, *vd)) return GRXDNN_STATUS_INVALID_VALUE;
  if (qd->batch != kd->batch || qd->headDim != kd->headDim) return GRXDNN_STATUS_INVALID_VALUE;
  if (qd->batch == 0 || qd->heads == 0 || qd->seq == 0) return GRXDNN_STATUS_SUCCESS;
  if (!q || !k || !v || !o) return GRXDNN_STATUS_INVALID_VALUE;
  if (!(scale > 0.0f) || isinf(scale)) return GRXDNN_STATUS_INVALID_VALUE;  // softmax scale must be finite, > 0
  if (causal && qd->seq != kd->seq) return GRXDNN_STATUS_NOT_SUPPORTED;
  if (kd->seq == 0) return GRXDNN_STATUS_NOT_SUPPORTED;
  for (auto* d : all)
    if (d->dtype != GRX_R_16BF) return GRXDNN_STATUS_NOT_SUPPORTED;
  if (qd->headDim != 128 || qd->heads != kd->heads) return GRXDNN_STATUS_NOT_SUPPORTED;
  auto& ctx = *reinterpret_cast<grxdnnContext*>(handle);
  grxdnnStatus_t s = ensure(ctx, true);
  if (s != GRXDNN_STATUS_SUCCESS) return s;
  grx::AttnArgs a{};
  a.batch = qd->batch;
  a.heads = qd->heads;
  a.seq_q = qd->seq;
  a.seq_k = kd->seq;
  a.q = q; a.q_sb = qd->strideBatch; a.q_sh = qd->strideHead; a.q_ss = qd->strideSeq;
  a.k = k; a.k_sb = kd->strideBatch; a.k_sh = kd->strideHead; a.k_ss = kd->strideSeq;
  a.v = v; a.v_sb = vd->strideBatch; a.v_sh = vd->strideHead; a.v_ss = vd->strideSeq;
  a.o = o; a.o_sb = od->strideBatch; a.o_sh = od->strideHead; a.o_ss = od->strideSeq;
  a.lse = lse;
  a.scale = scale;
  a.causal = causal ? 1 : 0;
  return from_cuda(grx::launch_attention_fwd(a, ctx.dev.num_sms, ctx.stream));
}

grxdnnStatus_t grxdnnAttentionBackward(grxdnnHandle_t handle, const grxdnnAttnTensor_t* qd, const void* q,
                                       const grxdnnAttnTensor_t* kd, const void* k, const grxdnnAttnTensor_t* vd,
                                       const void* v, const grxdnnAttnTensor_t* od, const void* o,
                                       const grxdnnAttnTensor_t* dod, const void* dout, const float* lse, float scale,
                                       int causal, const grxdnnAttnTensor_t* dqd, void* dq,
                                       const grxdnnAttnTensor_t* dkd, void* dk, const grxdnnAttnTensor_t* dvd,
                                       void* dv) {
  if (!handle) return GRXDNN_STATUS_NOT_INITIALIZED;
  if (!qd || !kd || !vd || !od || !dod || !dqd || !dkd || !dvd) return GRXDNN_STATUS_INVALID_VALUE;
  const grxdnnAttnTensor_t* all[8] = {qd, kd, vd, od, dod, dqd, dkd, dvd};
  for (auto* d : all)
    if (d->batch < 0 || d->heads < 0 || d->seq < 0 || d->headDim <= 0 || d->strideSeq < d->headDim)
      return GRXDNN_STATUS_INVALID_VALUE;
  if (!same_shape(*qd, *od) || !same_shape(*qd, *dod) || !same_shape(*qd, *dqd) || !same_shape(*kd, *vd) ||
      !same_shape(*kd, *dkd) || !same_shape(*kd, *dvd))
    return GRXDNN_STATUS_INVALID_VALUE;
  if (qd->batch != kd->batch || qd->headDim != kd->headDim) return GRXDNN_STATUS_INVALID_VALUE;
  if (qd->batch == 0 || qd->heads == 0 || qd->seq == 0) return GRXDNN_STATUS_SUCCESS;
  if (!q || !k || !v || !o || !dout || !lse || !dq || !dk || !dv) return GRXDNN_STATUS_INVALID_VALUE;
  if (!(scale > 0.0f) || isinf(scale)) return GRXDNN_STATUS_INVALID_VALUE;
  if (causal && qd->seq != kd->seq) return GRXDNN_STATUS_NOT_SUPPORTED;
  if (kd->seq == 0) return GRXDNN_STATUS_NOT_SUPPORTED;
  for (auto* d : all)
    if (d->dtype != GRX_R_16BF) return GRXDNN_STATUS_NOT_SUPPORTED;
  if (qd->headDim != 128 || qd->heads != kd->heads) return GRXDNN_STATUS_NOT_SUPPORTED;
  auto& ctx = *reinterpret_cast<grxdnnContext*>(handle);
  grxdnnStatus_t s = ensure(ctx, true);
  if (s != GRXDNN_STATUS_SUCCESS) return s;
  grx::AttnBwdArgs a{};
  a.batch = qd->batch;
  a.heads = qd->heads;
  a.seq_q = qd->seq;
  a.seq_k = kd->seq;
  a.q = q; a.q_sb = qd->strideBatch; a.q_sh = qd->strideHead; a.q_ss = qd->strideSeq;
  a.k = k; a.k_sb = kd->strideBatch; a.k_sh = kd->strideHead; a.k_ss = kd->strideSeq;
  a.v = v; a.v_sb = vd->strideBatch; a.v_sh = vd->strideHead; a.v_ss = vd->strideSeq;
  a.o = o; a.o_sb = od->strideBatch; a.o_sh = od->strideHead; a.o_ss = od->strideSeq;
  a.dout = dout; a.do_sb = dod->strideBatch; a.do_sh = dod->strideHead; a.do_ss = dod->strideSeq;
  a.lse = lse;
  a.dq = dq; a.dq_sb = dqd->strideBatch; a.dq_sh = dqd->strideHead; a.dq_ss = dqd->strideSeq;
  a.dk = dk; a.dk_sb = dkd->strideBatch; a.dk_sh = dkd->strideHead; a.dk_ss = dkd->strideSeq;
  a.dv = dv; a.dv_sb = dvd->strideBatch; a.dv_sh = dvd->strideHead; a.dv_ss = dvd->strideSeq;
  a.scale = scale;
  a.causal = causal ? 1 : 0;
  a.err_word = ctx.dev.err_word;
  a.timeout_ns = grx::wait_timeout_ns();
  const size_t need = grx::attention_bwd_workspace_bytes(a);
  void* ws = workspace(ctx, need);
  if (!ws) return GRXDNN_STATUS_ALLOC_FAILED;
  return from_cuda(grx::launch_attention_bwd(a, ws, need, ctx.stream));
}

grxdnnStatus_t grxdnnConvOutputDims(const grxdnnConvDesc_t* d, int* p, int* q) {
  if (!d || !p || !q) return GRXDNN_STATUS_INVALID_VALUE;
  if (d->h <= 0 || d->w <= 0 || d->r <= 0 || d->s <= 0 || d->padH < 0 || d->padW < 0 || d->strideH < 1 ||
      d->strideW < 1 || d->dilationH < 1 || d->dilationW < 1)
    return GRXDNN_STATUS_INVALID_VALUE;
  const long long eh = (long long)d->h + 2LL * d->padH - (long long)d->dilationH * (d->r - 1) - 1;
  const long long ew = (long long)d->w + 2LL * d->padW - (long long)d->dilationW * (d->s - 1) - 1;
  if (eh < 0 || ew < 0) return GRXDNN_STATUS_INVALID_VALUE;
  *p = (int)(eh / d->strideH + 1);
  *q = (int)(ew / d->strideW + 1);
  return GRXDNN_STATUS_SUCCESS;
}

grxdnnStatus_t grxdnnConv2dForward(grxdnnHandle_t handle, const grxdnnConvDesc_t* d, const void* x,
                                   grxDataType_t xType, const void* w, grxDataType_t wType, const float* alpha,
                                   const float* beta, const float* bias, int activation, void* y,
                                   grxDataType_t yType) {
  if (!handle) return GRXDNN_STATUS_NOT_INITIALIZED;
  if (!d) return GRXDNN_STATUS_INVALID_VALUE;
  int P = 0, Q = 0;
  if (d->n < 0 || d->c <= 0 || d->k <= 0) return GRXDNN_STATUS_INVALID_VALUE;
  grxdnnStatus_t s = grxdnnConvOutputDims(d, &P, &Q);
  if (s != GRXDNN_STATUS_SUCCESS) return s;
  if ((unsigned)activation > 3u) return GRXDNN_STATUS_INVALID_VALUE;
  if (d->n == 0) return GRXDNN_STATUS_SUCCESS;
  if (!x || !w || !y) return GRXDNN_STATUS_INVALID_VALUE;
  const int in_dt = xType == GRX_R_16BF ? 1 : xType == GRX_R_32F ? 0 : -1;
  const int out_dt = yType == GRX_R_16BF ? 1 : yType == GRX_R_32F ? 0 : -1;
  if (in_dt < 0 || out_dt < 0 || wType != xType || (in_dt == 0 && out_dt != 0)) return GRXDNN_STATUS_NOT_SUPPORTED;
  const float al = alpha ? *alpha : 1.f, be = beta ? *beta : 0.f;
  auto& ctx = *reinterpret_cast<grxdnnContext*>(handle);
  s = ensure(ctx, false);
  if (s != GRXDNN_STATUS_SUCCESS) return s;
  if (in_dt == 1 && d->c % 64 == 0 && ctx.dev.cc_major == 10) {
    grx::TcConvLaunch L{};
    L.out = out_dt == 1 ? grx::kOutBF16 : grx::kOutF32;
    L.x = x;
    L.w = w;
    L.n = d->n; L.h = d->h; L.wd = d->w; L.c = d->c; L.k = d->k; L.r = d->r; L.s = d->s; L.p = P; L.q = Q;
    L.pad_h = d->padH; L.pad_w = d->padW; L.stride_h = d->strideH; L.stride_w = d->strideW;
    L.dil_h = d->dilationH; L.dil_w = d->dilationW;
    grx::TcGemmParams& e = L.p_epi;
    e.alpha = al;
    e.beta = be;
    e.beta_nonzero = be != 0.f ? 1 : 0;
    e.c = y;
    e.ldc = d->k;
    e.bias = bias;
    e.bias_rows = 1;
    e.act = activation;
    e.err_word = ctx.dev.err_word;
    e.timeout_ns = grx::wait_timeout_ns();
    e.group_m = 16;
    const cudaError_t err = grx::launch_tc_conv(L, ctx.dev.num_sms, ctx.stream);
    if (err != cudaErrorNotSupported) return from_cuda(err);
    cudaGetLastError();  // not expressible as TMA boxes: the direct kernel takes it
  }
  grx::ConvArgs a{};
  a.n = d->n; a.h = d->h; a.w = d->w; a.c = d->c; a.k = d->k; a.r = d->r; a.s = d->s; a.p = P; a.q = Q;
  a.pad_h = d->padH; a.pad_w = d->padW; a.stride_h = d->strideH; a.stride_w = d->strideW;
  a.dil_h = d->dilationH; a.dil_w = d->dilationW;
  a.in_dtype = in_dt;
  a.out_dtype = out_dt;
  a.x = x; a.filt = w; a.y = y;
  a.bias = bias;
  a.alpha = al;
  a.beta = be;
  a.act = activation;
  return from_cuda(grx::launch_conv2d_direct(a, ctx.dev.num_sms, ctx.stream));
}

grxdnnStatus_t grxdnnPoolingOutputDims(const grxdnnPoolDesc_t* d, int* p, int* q) {
  if (!d || !p || !q) return GRXDNN_STATUS_INVALID_VALUE;
  grxdnnConvDesc_t c{};
  c.h = d->h; c.w = d->w; c.r = d->r; c.s = d->s; c.padH = d->padH; c.padW = d->padW;
  c.strideH = d->strideH; c.strideW = d->strideW; c.dilationH = 1; c.dilationW = 1;
  return grxdnnConvOutputDims(&c, p, q);
}

grxdnnStatus_t grxdnnPooling2dForward(grxdnnHandle_t handle, const grxdnnPoolDesc_t* d, const void* x,
                                      grxDataType_t xType, void* y, grxDataType_t yType) {
  if (!handle) return GRXDNN_STATUS_NOT_INITIALIZED;
  if (!d) return GRXDNN_STATUS_INVALID_VALUE;
  int P = 0, Q = 0;
  if (d->n < 0 || d->c <= 0 || (unsigned)d->mode > 2u) return GRXDNN_STATUS_INVALID_VALUE;
  grxdnnStatus_t s = grxdnnPoolingOutputDims(d, &P, &Q);
  if (s != GRXDNN_STATUS_SUCCESS) return s;
  if (d->n == 0) return GRXDNN_STATUS_SUCCESS;
  if (!x || !y) return GRXDNN_STATUS_INVALID_VALUE;
  if (xType != yType || norm_dtype(xType) < 0) return GRXDNN_STATUS_NOT_SUPPORTED;
  auto& ctx = *reinterpret_cast<grxdnnContext*>(handle);
  s = ensure(ctx, false);
  if (s != GRXDNN_STATUS_SUCCESS) return s;
  grx::PoolArgs a{};
  a.n = d->n; a.h = d->h; a.w = d->w; a.c = d->c; a.r = d->r; a.s = d->s; a.p = P; a.q = Q;
  a.pad_h = d->padH; a.pad_w = d->padW; a.stride_h = d->strideH; a.stride_w = d->strideW;
  a.mode = (int)d->mode;
  a.dtype = norm_dtype(xType);
  a.x = x;
  a.y = y;
  return from_cuda(grx::launch_pool2d(a, ctx.dev.num_sms, ctx.stream));
}

grxdnnStatus_t grxdnnGetExecutionStatus(grxdnnHandle_t handle) {
  if (!handle) return GRXDNN_STATUS_NOT_INITIALIZED;
  auto* ctx = reinterpret_cast<grxdnnContext*>(handle);
  std::lock_guard<std::mutex> lock(ctx->mutex);
  const int code = grx::take_error(ctx->dev, ctx->stream);
  return code == 0 ? GRXDNN_STATUS_SUCCESS : GRXDNN_STATUS_EXECUTION_FAILED;
}

}  // extern "C"
