/* grxcp-b200 -- grxDNN: transformer primitives on B200 (sm_100a).
 *
 * The reference plans a grxDNN library beside grxBLAS (docs/designs/
 * grxcp_architecture.md:594, docs/designs/grxcp_roadmap.md:860-876,
 * src/libs/CMakeLists.txt:12) but ships no header, code or tests for it. This
 * header is therefore new; it follows grxBLAS's conventions so a caller of one
 * knows the other: an opaque handle bound to a stream, status codes with the
 * same values as grxblasStatus_t, device pointers for tensors, host values for
 * scalars, no host synchronisation inside a call, and refusal (never a silent
 * fallback) for anything the kernels do not implement.
 */
#ifndef GRXDNN_H
#define GRXDNN_H

#include "grx_runtime.h"
#include "grx_types.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct grxdnnContext* grxdnnHandle_t;

typedef enum {
  GRXDNN_STATUS_SUCCESS          = 0,
  GRXDNN_STATUS_NOT_INITIALIZED  = 1,
  GRXDNN_STATUS_ALLOC_FAILED     = 2,
  GRXDNN_STATUS_INVALID_VALUE    = 3,
  GRXDNN_STATUS_ARCH_MISMATCH    = 4,
  GRXDNN_STATUS_EXECUTION_FAILED = 5,
  GRXDNN_STATUS_NOT_SUPPORTED    = 6,
  GRXDNN_STATUS_INTERNAL_ERROR   = 7
} grxdnnStatus_t;

const char*    grxdnnGetStatusString(grxdnnStatus_t s);
grxdnnStatus_t grxdnnCreate(grxdnnHandle_t* handle);
grxdnnStatus_t grxdnnDestroy(grxdnnHandle_t handle);
grxdnnStatus_t grxdnnSetStream(grxdnnHandle_t handle, grxStream_t stream);
grxdnnStatus_t grxdnnGetStream(grxdnnHandle_t handle, grxStream_t* stream);

/* RMSNorm forward over the last dimension of a [rows, hidden] matrix:
 *   y[r, c] = x[r, c] * rsqrt(mean_c(x[r, :]^2) + eps) * gamma[c]
 * Statistics in fp32. x/y: GRX_R_16BF (or GRX_R_16F, GRX_R_32F, same type for
 * both); ldx/ldy are row pitches in elements (>= hidden). gamma is fp32
 * [hidden]. rstd (fp32 [rows]) may be NULL. rows == 0 is SUCCESS. */
grxdnnStatus_t grxdnnRMSNormForward(grxdnnHandle_t handle, int rows, int hidden,
                                    const void* x, grxDataType_t xType, long long ldx,
                                    const float* gamma, float eps,
                                    void* y, grxDataType_t yType, long long ldy,
                                    float* rstd);

/* LayerNorm forward over the last dimension:
 *   y[r, c] = (x[r, c] - mu_r) * rsqrt(var_r + eps) * gamma[c] + beta[c]
 * with population variance, statistics in fp32. beta may be NULL (no shift);
 * mean and rstd (fp32 [rows]) may be NULL. Types and pitches as RMSNorm. */
grxdnnStatus_t grxdnnLayerNormForward(grxdnnHandle_t handle, int rows, int hidden,
                                      const void* x, grxDataType_t xType, long long ldx,
                                      const float* gamma, const float* beta, float eps,
                                      void* y, grxDataType_t yType, long long ldy,
                                      float* mean, float* rstd);

/* RMSNorm backward (no counterpart in the reference, whose grxDNN is planned
 * only): with r = rstd of the row and H = hidden,
 *   dx[r, c] = r gamma[c] dy[r, c] - x[r, c] r^3 (sum_c dy gamma x) / H
 *   dgamma[c] = sum_rows dy[r, c] x[r, c] r
 * in fp32. dy, x and dx share one type (as the forward's x/y) and have row
 * pitches lddy/ldx/lddx >= hidden. rstd is the forward's fp32 [rows] output,
 * or NULL to recompute it from x with eps. dgamma (fp32 [hidden]) is
 * overwritten, summed in a fixed order (bit-reproducible); NULL skips it.
 * rows == 0 writes dgamma = 0. Uses handle-owned scratch (grown on demand,
 * stream-ordered) for dgamma partial sums. */
grxdnnStatus_t grxdnnRMSNormBackward(grxdnnHandle_t handle, int rows, int hidden,
                                     const void* dy, grxDataType_t dyType, long long lddy,
                                     const void* x, grxDataType_t xType, long long ldx,
                                     const float* gamma, const float* rstd, float eps,
                                     void* dx, grxDataType_t dxType, long long lddx,
                                     float* dgamma);

/* LayerNorm backward (no counterpart in the reference): with xh = (x - mu) r,
 *   dx = r (dy gamma - mean_c(dy gamma) - xh mean_c(dy gamma xh))
 *   dgamma[c] = sum_rows dy xh,   dbeta[c] = sum_rows dy
 * mean and rstd are the forward's outputs (both given, or both NULL to
 * recompute from x with eps). dgamma / dbeta may each be NULL. Otherwise as
 * grxdnnRMSNormBackward. */
grxdnnStatus_t grxdnnLayerNormBackward(grxdnnHandle_t handle, int rows, int hidden,
                                       const void* dy, grxDataType_t dyType, long long lddy,
                                       const void* x, grxDataType_t xType, long long ldx,
                                       const float* gamma, const float* mean, const float* rstd,
                                       float eps, void* dx, grxDataType_t dxType, long long lddx,
                                       float* dgamma, float* dbeta);

/* Softmax over the last dimension of a [rows, cols] matrix:
 *   y[r, c] = exp(x[r, c] - max_c x[r, :]) / sum_c exp(x[r, c] - max_c x[r, :])
 * in fp32. x/y of the same type (GRX_R_16BF, GRX_R_16F or GRX_R_32F), row
 * pitches ldx/ldy >= cols. rows == 0 is SUCCESS. y may alias x (in place,
 * with ldy == ldx). */
grxdnnStatus_t grxdnnSoftmaxForward(grxdnnHandle_t handle, int rows, int cols,
                                    const void* x, grxDataType_t xType, long long ldx,
                                    void* y, grxDataType_t yType, long long ldy);

/* GELU over n contiguous elements, y = x * Phi(x): GRXDNN_GELU_ERF uses the
 * erf form of the Gaussian CDF, GRXDNN_GELU_TANH its tanh approximation.
 * fp32 arithmetic; x and y of the same type, may alias. */
typedef enum {
  GRXDNN_GELU_ERF  = 0,
  GRXDNN_GELU_TANH = 1
} grxdnnGeluMode_t;

grxdnnStatus_t grxdnnGeluForward(grxdnnHandle_t handle, long long n,
                                 const void* x, grxDataType_t xType,
                                 void* y, grxDataType_t yType, grxdnnGeluMode_t mode);

/* A [batch, heads, seq, headDim] tensor with element strides; the headDim
 * stride is 1. */
typedef struct {
  int           batch, heads, seq, headDim;
  long long     strideBatch, strideHead, strideSeq;
  grxDataType_t dtype;
} grxdnnAttnTensor_t;

/* Fused scaled-dot-product attention forward:
 *   O = softmax(scale * Q K^T + mask) V,   lse = log(sum exp(scale * Q K^T + mask))
 * per (batch, head). causal != 0 masks key j > query i (requires equal q/k
 * sequence lengths). dtype GRX_R_16BF (Q, K, V, O alike), headDim 128, equal
 * head counts. lse is fp32 [batch, heads, seqQ] contiguous (natural log), may
 * be NULL. scale must be finite and > 0. The softmax runs in fp32, both
 * contractions accumulate in fp32 on the tensor cores. */
grxdnnStatus_t grxdnnAttentionForward(grxdnnHandle_t handle,
                                      const grxdnnAttnTensor_t* qDesc, const void* q,
                                      const grxdnnAttnTensor_t* kDesc, const void* k,
                                      const grxdnnAttnTensor_t* vDesc, const void* v,
                                      const grxdnnAttnTensor_t* oDesc, void* o,
                                      float scale, int causal, float* lse);

/* Synchronises the handle's stream; EXECUTION_FAILED if a kernel launched
 * through this handle gave up on a bounded wait since the last query. */
/* Attention backward (no counterpart in the reference): gradients of
 * grxdnnAttentionForward. From Q, K, V, the forward's O and LSE, and dO:
 *   P = exp(scale Q K^T - LSE) (masked as in the forward), Delta = rowsum(dO * O),
 *   dV = P^T dO,  dS = P * (dO V^T - Delta),  dK = scale dS^T Q,  dQ = scale dS K.
 * fp32 accumulation, bf16 outputs; every tensor bf16 with headDim 128 in its
 * own descriptor (dq/dO/o shaped as q, dk/dv shaped as k), lse fp32
 * [batch, heads, seq_q] as the forward wrote it. Bit-reproducible (no
 * atomics). Uses handle-owned scratch (4 bytes per query row). Argument rules
 * as grxdnnAttentionForward. */
grxdnnStatus_t grxdnnAttentionBackward(grxdnnHandle_t handle,
                                       const grxdnnAttnTensor_t* qDesc, const void* q,
                                       const grxdnnAttnTensor_t* kDesc, const void* k,
                                       const grxdnnAttnTensor_t* vDesc, const void* v,
                                       const grxdnnAttnTensor_t* oDesc, const void* o,
                                       const grxdnnAttnTensor_t* dODesc, const void* dO,
                                       const float* lse, float scale, int causal,
                                       const grxdnnAttnTensor_t* dQDesc, void* dQ,
                                       const grxdnnAttnTensor_t* dKDesc, void* dK,
                                       const grxdnnAttnTensor_t* dVDesc, void* dV);

/* 2-D convolution (planned in the reference's grxDNN as "conv2d (implicit
 * GEMM)", never implemented there): NHWC input x [n, h, w, c], KRSC filters
 * [k, r, s, c], NHWC output y [n, p, q, k] with
 *   p = (h + 2 padH - dilationH (r - 1) - 1) / strideH + 1   (q likewise),
 *   y = act(alpha * conv(x, w) + beta * y + bias[k]).
 * alpha / beta are host pointers (NULL: 1 / 0; beta == 0 never reads y).
 * bias (fp32 [k]) may be NULL; activation as grxblasActivation_t (0 none,
 * 1 ReLU, 2 GELU tanh, 3 GELU erf). Types: x and w both GRX_R_16BF (y bf16 or
 * fp32) or both GRX_R_32F (y fp32). bf16 with c a multiple of 64 runs as an
 * implicit GEMM on the tensor cores; other shapes run a direct kernel. */
typedef struct {
  int n, h, w, c;
  int k, r, s;
  int padH, padW, strideH, strideW, dilationH, dilationW;
} grxdnnConvDesc_t;

grxdnnStatus_t grxdnnConvOutputDims(const grxdnnConvDesc_t* desc, int* p, int* q);
grxdnnStatus_t grxdnnConv2dForward(grxdnnHandle_t handle, const grxdnnConvDesc_t* desc,
                                   const void* x, grxDataType_t xType,
                                   const void* w, grxDataType_t wType,
                                   const float* alpha, const float* beta,
                                   const float* bias, int activation,
                                   void* y, grxDataType_t yType);

/* 2-D pooling over NHWC (planned in the reference's grxDNN, never
 * implemented): windows r x s at the given strides and zero-based padding;
 * MAX (a window wholly in the padding gives 0), AVG_INCLUDE_PAD (divide by
 * r s) or AVG_EXCLUDE_PAD (divide by the in-image taps). x and y share one
 * type (GRX_R_16BF, GRX_R_16F, GRX_R_32F); y is [n, p, q, c] with p, q as
 * for conv with dilation 1. */
typedef enum {
  GRXDNN_POOL_MAX = 0,
  GRXDNN_POOL_AVG_INCLUDE_PAD = 1,
  GRXDNN_POOL_AVG_EXCLUDE_PAD = 2
} grxdnnPoolMode_t;

typedef struct {
  int n, h, w, c;
  int r, s;
  int padH, padW, strideH, strideW;
  grxdnnPoolMode_t mode;
} grxdnnPoolDesc_t;

grxdnnStatus_t grxdnnPoolingOutputDims(const grxdnnPoolDesc_t* desc, int* p, int* q);
grxdnnStatus_t grxdnnPooling2dForward(grxdnnHandle_t handle, const grxdnnPoolDesc_t* desc,
                                      const void* x, grxDataType_t xType,
                                      void* y, grxDataType_t yType);

/* Softmax backward (no counterpart in the reference): from the forward's
 * output y and the gradient dy, dx[r, c] = y[r, c] (dy[r, c] - sum_c dy y),
 * fp32 math; y, dy, dx of one type (GRX_R_16BF, GRX_R_16F, GRX_R_32F) with
 * row pitches >= cols. rows == 0 is SUCCESS. dx may alias dy or y (in place,
 * with equal pitches). */
grxdnnStatus_t grxdnnSoftmaxBackward(grxdnnHandle_t handle, int rows, int cols,
                                     const void* y, grxDataType_t yType, long long ldy,
                                     const void* dy, grxDataType_t dyType, long long lddy,
                                     void* dx, grxDataType_t dxType, long long lddx);

/* GELU backward (no counterpart in the reference): dx = dy * GELU'(x) for
 * the same mode as grxdnnGeluForward; n contiguous elements, x, dy, dx of
 * one type. n == 0 is SUCCESS. dx may alias dy or x. */
grxdnnStatus_t grxdnnGeluBackward(grxdnnHandle_t handle, long long n, const void* x, const void* dy,
                                  void* dx, grxDataType_t type, grxdnnGeluMode_t mode);

grxdnnStatus_t grxdnnGetExecutionStatus(grxdnnHandle_t handle);

#ifdef __cplusplus
}
#endif

#endif /* GRXDNN_H */
