// grxBLAS host library for B200.
//
// Replaces src/libs/grxblas/grxblas.cpp of the reference. The argument
// validation, its ORDER, and the status each refusal returns are the
// reference's (cited per function); what happens after validation is new: no
// module loading or descriptor-slot programming, but a launch of a sm_100a
// kernel compiled into this library, on the handle's stream, with no host
// synchronisation.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <limits.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <atomic>
#include <mutex>
#include <string>

#include "gemm_tc.cuh"
#include "grx/grxblas.h"
#include "host_common.h"
#include "kernels.h"

struct grxblasContext {
  cudaStream_t stream = nullptr;
  std::mutex mutex;
  int slot_a = 0, slot_b = 1;
  grxCycleSlot* probe = nullptr;
  int probe_capacity = 0;
  grxblasEpilogue_t epi{};
  bool has_epi = false;
  void* ws_user = nullptr;
  size_t ws_user_bytes = 0;
  void* ws_own = nullptr;
  size_t ws_own_bytes = 0;
  grx::DeviceState dev;
  bool loaded = false;
  int n_peers = 0;
  void* peers[grx::kMaxPeers] = {};
};

namespace {

std::mutex g_path_mutex;
std::string g_kernel_path;  // grxblasSetKernelPath

grxblasStatus_t from_cuda(cudaError_t e) {
  switch (e) {
    case cudaSuccess: return GRXBLAS_STATUS_SUCCESS;
    case cudaErrorMemoryAllocation: return GRXBLAS_STATUS_ALLOC_FAILED;
    case cudaErrorInvalidValue: return GRXBLAS_STATUS_INVALID_VALUE;
    case cudaErrorNotSupported: return GRXBLAS_STATUS_NOT_SUPPORTED;
    case cudaErrorNoKernelImageForDevice:
    case cudaErrorInvalidDeviceFunction: return GRXBLAS_STATUS_ARCH_MISMATCH;
    default: return GRXBLAS_STATUS_EXECUTION_FAILED;
  }
}

// Configured-path rule of reference grxblas.cpp:33-58 / grxblas.h:214-227: a
// configured path (call, then $GRXBLAS_KERNEL_PATH) must name the file the
// kernels live in -- this library -- or its directory; no fallback past it.
bool kernel_path_ok() {
  if (grx::fault_injected("module")) return false;
  std::string cfg;
  {
    std::lock_guard<std::mutex> lock(g_path_mutex);
    cfg = g_kernel_path;
  }
  if (cfg.empty()) {
    const char* env = getenv("GRXBLAS_KERNEL_PATH");
    if (env) cfg = env;
  }
  if (cfg.empty()) return true;
  return grx::path_names_library(cfg.c_str());
}

// First-use set-up of a handle (reference ensure_hgemm, grxblas.cpp:188-307,
// minus the module load and shape-kernel round trip: the tile and type set are
// constants of this build). Called with ctx.mutex held.
grxblasStatus_t ensure_locked(grxblasContext& ctx, bool need_tensor) {
  if (!kernel_path_ok()) return GRXBLAS_STATUS_NOT_INITIALIZED;
  const int rc = grx::ensure_device(ctx.dev);
  if (rc == 1) return GRXBLAS_STATUS_NOT_INITIALIZED;
  if (rc == 2) return GRXBLAS_STATUS_ALLOC_FAILED;
  if (need_tensor && ctx.dev.cc_major != 10) return GRXBLAS_STATUS_ARCH_MISMATCH;
  ctx.loaded = true;
  return GRXBLAS_STATUS_SUCCESS;
}

grxblasStatus_t ensure(grxblasContext& ctx, bool need_tensor) {
  std::lock_guard<std::mutex> lock(ctx.mutex);
  return ensure_locked(ctx, need_tensor);
}

bool is_int(float v) {
  return v >= -2147483648.0f && v < 2147483648.0f && v == (float)(int32_t)v;
}

// Grow-only stream-ordered workspace owned by the handle.
void* workspace(grxblasContext& ctx, size_t bytes) {
  if (bytes == 0) return nullptr;
  if (ctx.ws_user && ctx.ws_user_bytes >= bytes) return ctx.ws_user;
  if (ctx.ws_own_bytes >= bytes) return ctx.ws_own;
  if (grx::fault_injected("alloc")) return nullptr;
  if (ctx.ws_own) cudaFreeAsync(ctx.ws_own, ctx.stream);
  ctx.ws_own = nullptr;
  ctx.ws_own_bytes = 0;
  void* p = nullptr;
  if (cudaMallocAsync(&p, bytes, ctx.stream) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  ctx.ws_own = p;
  ctx.ws_own_bytes = bytes;
  return p;
}

struct TypeCase {
  int kind, out, a_fmt, es;
};

// Accepted (Atype, Btype, Ctype) triples. Returns false for anything else.
bool classify(grxDataType_t at, grxDataType_t bt, grxDataType_t ct, TypeCase& tc) {
  if (at != bt) return false;
  switch (at) {
    case GRX_R_16F:
      if (ct == GRX_R_32F) tc = {grx::kKindF16, grx::kOutF32, 0, 2};
      else if (ct == GRX_R_16F) tc = {grx::kKindF16, grx::kOutF16, 0, 2};
      else return false;
      return true;
    case GRX_R_16BF:
      if (ct == GRX_R_32F) tc = {grx::kKindF16, grx::kOutF32, 1, 2};
      else if (ct == GRX_R_16BF) tc = {grx::kKindF16, grx::kOutBF16, 1, 2};
      else return false;
      return true;
    case GRX_R_8I:
      if (ct == GRX_R_32I) tc = {grx::kKindI8, grx::kOutS32, 1, 1};
      else if (ct == GRX_R_16BF) tc = {grx::kKindI8, grx::kOutBF16, 1, 1};
      else if (ct == GRX_R_32F) tc = {grx::kKindI8, grx::kOutF32, 1, 1};
      else return false;
      return true;
    case GRX_R_8F_E4M3:
      if (ct == GRX_R_16BF) tc = {grx::kKindF8, grx::kOutBF16, 0, 1};
      else if (ct == GRX_R_32F) tc = {grx::kKindF8, grx::kOutF32, 0, 1};
      else return false;
      return true;
    default: return false;
  }
}

void say_types_once() {
  static std::atomic<bool> said{false};
  if (said.exchange(true)) return;
  fprintf(stderr,
          "grxblas: grxblasGemmEx accepts (A, B, C) = (16F,16F,32F|16F), (16BF,16BF,32F|16BF),\n"
          "         (8I,8I,32I|16BF|32F) and (8F_E4M3,8F_E4M3,16BF|32F) on this device\n"
          "         (query grxblasGetTensorTypes); other pairings are refused, never emulated.\n");
}

long long round_up(long long v, long long a) { return (v + a - 1) / a * a; }

// Bytes of packed copy an operand needs when it cannot be fed to TMA as stored.
size_t pack_bytes(int rows, int k, int es, int batch_eff) {
  const long long ldp = round_up(k, 16 / es);
  return (size_t)round_up((long long)batch_eff * rows * ldp * es, 256);
}

struct OperandPlan {
  const void* ptr;
  long long ld, stride;
  int mn_major;
  bool pack;
  int batch_eff;
};

OperandPlan plan_operand(const void* ptr, int mn_major, long long ld, long long stride, int es, int batch) {
  OperandPlan o{ptr, ld, stride, mn_major, false, 1};
  o.batch_eff = (batch > 1 && stride != 0) ? batch : 1;
  o.pack = !grx::tma_operand_ok(ptr, ld, stride, es, batch);
  return o;
}

grxblasStatus_t gemm_ex_impl(grxblasHandle_t handle, grxblasOperation_t transa, grxblasOperation_t transb, int m,
                             int n, int k, const float* alpha, const void* A, grxDataType_t Atype, int lda,
                             long long strideA, const void* B, grxDataType_t Btype, int ldb, long long strideB,
                             const float* beta, void* C, grxDataType_t Ctype, int ldc, long long strideC,
                             int batch, long long col0 = 0) {
  // Order and codes: reference grxblas.cpp:506-524 (GemmEx) and :882-897
  // (the batch rules of sgemm_batched).
  if (!handle) return GRXBLAS_STATUS_NOT_INITIALIZED;
  if (!alpha || !beta) return GRXBLAS_STATUS_INVALID_VALUE;
  if (m < 0 || n < 0 || k < 0) return GRXBLAS_STATUS_INVALID_VALUE;
  if (batch < 0) return GRXBLAS_STATUS_INVALID_VALUE;
  if (m == 0 || n == 0 || batch == 0) return GRXBLAS_STATUS_SUCCESS;
  if (k > 0 && (!A || !B)) return GRXBLAS_STATUS_INVALID_VALUE;
  if (!C) return GRXBLAS_STATUS_INVALID_VALUE;
  const bool ta = (transa == GRXBLAS_OP_T);
  const bool tb = (transb == GRXBLAS_OP_T);
  const int min_lda = ta ? k : m;
  const int min_ldb = tb ? n : k;
  if (lda < min_lda || ldb < min_ldb || ldc < m) return GRXBLAS_STATUS_INVALID_VALUE;

  auto& ctx = *reinterpret_cast<grxblasContext*>(handle);
  std::lock_guard<std::mutex> lock(ctx.mutex);
  grxblasStatus_t st = ensure_locked(ctx, true);
  if (st != GRXBLAS_STATUS_SUCCESS) return st;

  // Type check after set-up, as the reference does (grxblas.cpp:552-575).
  TypeCase tc;
  if (!classify(Atype, Btype, Ctype, tc)) {
    say_types_once();
    return GRXBLAS_STATUS_NOT_SUPPORTED;
  }
  // Integer pairing: alpha/beta must be exact integers (grxblas.cpp:580-584).
  if (tc.out == grx::kOutS32) {
    if (!is_int(*alpha) || !is_int(*beta)) return GRXBLAS_STATUS_INVALID_VALUE;
    if (ctx.has_epi && (ctx.epi.bias || ctx.epi.scaleMode != GRXBLAS_SCALE_NONE))
      return GRXBLAS_STATUS_NOT_SUPPORTED;
  }
  grxblasEpilogue_t epi = ctx.has_epi ? ctx.epi : grxblasEpilogue_t{};
  if (col0 != 0) {
    // columns [col0, col0 + n) of a wider problem: per-column bias and scales start at col0
    if (epi.bias && !epi.biasOverRows)
      epi.bias = static_cast<const char*>(epi.bias) + col0 * (epi.biasType == GRX_R_16BF ? 2 : 4);
    if (epi.scaleMode == GRXBLAS_SCALE_ROWCOL && epi.scaleB) epi.scaleB += col0;
  }
  if (epi.scaleMode != GRXBLAS_SCALE_NONE && (!epi.scaleA || !epi.scaleB)) return GRXBLAS_STATUS_INVALID_VALUE;
  if ((unsigned)epi.scaleMode > 2u) return GRXBLAS_STATUS_INVALID_VALUE;
  if (epi.bias && epi.biasType != GRX_R_32F && epi.biasType != GRX_R_16BF) return GRXBLAS_STATUS_NOT_SUPPORTED;
  if ((unsigned)epi.activation > 3u) return GRXBLAS_STATUS_INVALID_VALUE;
  if (tc.out == grx::kOutS32 && ctx.has_epi && (epi.activation != GRXBLAS_ACT_NONE)) return GRXBLAS_STATUS_NOT_SUPPORTED;
  const int bias_bf16 = (epi.bias && epi.biasType == GRX_R_16BF) ? 1 : 0;

  if (ctx.n_peers > 0 && (k == 0 || tc.kind != grx::kKindF16)) return GRXBLAS_STATUS_NOT_SUPPORTED;
  if (k == 0) {
    // C = beta*C (+ bias): no product to form (reference test case "k = 0
    // scales C by beta", tests/libs/test_grxblas_ex.cpp:217).
    return from_cuda(grx::launch_gemm_k0(tc.out, C, ldc, strideC, m, n, batch, *beta, (int)*beta, epi.bias,
                                         bias_bf16, epi.strideBias, epi.biasOverRows ? 1 : 0, (int)epi.activation,
                                         ctx.stream));
  }

  OperandPlan pa = plan_operand(A, ta ? 0 : 1, lda, strideA, tc.es, batch);
  OperandPlan pb = plan_operand(B, tb ? 1 : 0, ldb, strideB, tc.es, batch);
  const size_t need_a = pa.pack ? pack_bytes(m, k, tc.es, pa.batch_eff) : 0;
  const size_t need_b = pb.pack ? pack_bytes(n, k, tc.es, pb.batch_eff) : 0;
  // Workspace: [packed A][packed B][split-K partials and counters]. The
  // split-K part is optional: without room for it the launch keeps the
  // whole-tile schedule.
  const size_t pack_total = (need_a + need_b + 255) & ~(size_t)255;
  const size_t need_sk = grx::tc_gemm_splitk_bytes(tc.kind, m, n, k, batch, ctx.dev.num_sms);
  uint8_t* sk_ws = nullptr;
  if (need_sk) {
    uint8_t* w = static_cast<uint8_t*>(workspace(ctx, pack_total + need_sk));
    if (w) sk_ws = w + pack_total;
  }
  if (need_a + need_b > 0) {
    uint8_t* ws = static_cast<uint8_t*>(workspace(ctx, sk_ws ? pack_total + need_sk : need_a + need_b));
    if (!ws) return GRXBLAS_STATUS_ALLOC_FAILED;
    const long long ldp = round_up(k, 16 / tc.es);
    if (pa.pack) {
      cudaError_t e = grx::launch_pack_kmajor(A, tc.es, pa.mn_major, lda, strideA, pa.batch_eff, m, k, ws, ldp,
                                              ctx.stream);
      if (e != cudaSuccess) return from_cuda(e);
      pa = OperandPlan{ws, ldp, (long long)m * ldp, 0, true, pa.batch_eff};
    }
    if (pb.pack) {
      uint8_t* wb = ws + need_a;
      cudaError_t e = grx::launch_pack_kmajor(B, tc.es, pb.mn_major, ldb, strideB, pb.batch_eff, n, k, wb, ldp,
                                              ctx.stream);
      if (e != cudaSuccess) return from_cuda(e);
      pb = OperandPlan{wb, ldp, (long long)n * ldp, 0, true, pb.batch_eff};
    }
  }

  grx::TcGemmLaunch L{};
  L.kind = tc.kind;
  L.out = tc.out;
  L.a_fmt = tc.a_fmt;
  L.a = pa.ptr;
  L.lda = pa.ld;
  L.stride_a = pa.batch_eff > 1 ? pa.stride : 0;
  L.a_mn_major = pa.mn_major;
  L.b = pb.ptr;
  L.ldb = pb.ld;
  L.stride_b = pb.batch_eff > 1 ? pb.stride : 0;
  L.b_mn_major = pb.mn_major;
  L.sk_ws = sk_ws;
  L.sk_ws_bytes = sk_ws ? need_sk : 0;
  grx::TcGemmParams& p = L.p;
  p.m = m;
  p.n = n;
  p.k = k;
  p.batch = batch;
  p.alpha = *alpha;
  p.beta = *beta;
  p.ialpha = (int)*alpha;
  p.ibeta = (int)*beta;
  p.beta_nonzero = (*beta != 0.0f) ? 1 : 0;
  p.c = C;
  p.ldc = ldc;
  p.stride_c = strideC;
  p.bias = epi.bias;
  p.bias_bf16 = bias_bf16;
  p.bias_rows = epi.biasOverRows ? 1 : 0;
  p.act = (int)epi.activation;
  p.stride_bias = epi.strideBias;
  p.scale_mode = (int)epi.scaleMode;
  p.scale_a = epi.scaleA;
  p.scale_b = epi.scaleB;
  p.stride_sa = epi.strideScaleA;
  p.stride_sb = epi.strideScaleB;
  p.err_word = ctx.dev.err_word;
  p.timeout_ns = grx::wait_timeout_ns();
  p.group_m = 16;
  p.n_peers = ctx.n_peers;
  for (int i = 0; i < ctx.n_peers; ++i) p.peers[i] = ctx.peers[i];
  // One probe slot per CTA of the launch, as the reference's GemmEx records
  // one per warp (grxblas.cpp:690-694); too few slots is INVALID_VALUE.
  p.probe = ctx.probe;
  p.probe_capacity = ctx.probe_capacity;
  return from_cuda(grx::launch_tc_gemm(L, ctx.dev.num_sms, ctx.stream));
}

}  // namespace

namespace grx {
grxblasStatus_t gemm_ex_columns(grxblasHandle_t handle, grxblasOperation_t transa, grxblasOperation_t transb, int m,
                                int n, int k, const float* alpha, const void* A, grxDataType_t Atype, int lda,
                                const void* B, grxDataType_t Btype, int ldb, const float* beta, void* C,
                                grxDataType_t Ctype, int ldc, long long col0) {
  return gemm_ex_impl(handle, transa, transb, m, n, k, alpha, A, Atype, lda, 0, B, Btype, ldb, 0, beta, C, Ctype, ldc,
                      0, 1, col0);
}
}  // namespace grx

extern "C" {

const char* grxblasGetStatusString(grxblasStatus_t s) {
  switch (s) {
    case GRXBLAS_STATUS_SUCCESS: return "success";
    case GRXBLAS_STATUS_NOT_INITIALIZED: return "library not initialized (no usable device, or a configured kernel path that is not this library)";
    case GRXBLAS_STATUS_ALLOC_FAILED: return "allocation failed";
    case GRXBLAS_STATUS_INVALID_VALUE: return "invalid argument";
    case GRXBLAS_STATUS_ARCH_MISMATCH: return "device lacks a required capability (sm_100 tensor cores)";
    case GRXBLAS_STATUS_EXECUTION_FAILED: return "kernel execution failed";
    case GRXBLAS_STATUS_NOT_SUPPORTED: return "not supported";
    case GRXBLAS_STATUS_INTERNAL_ERROR: return "internal error";
  }
  return "unknown status";
}

grxblasStatus_t grxblasCreate(grxblasHandle_t* handle) {
  if (!handle) return GRXBLAS_STATUS_INVALID_VALUE;
  *handle = reinterpret_cast<grxblasHandle_t>(new grxblasContext());
  return GRXBLAS_STATUS_SUCCESS;
}

grxblasStatus_t grxblasDestroy(grxblasHandle_t handle) {
  if (!handle) return GRXBLAS_STATUS_NOT_INITIALIZED;
  auto* ctx = reinterpret_cast<grxblasContext*>(handle);
  if (ctx->ws_own) {
    cudaFreeAsync(ctx->ws_own, ctx->stream);
    cudaStreamSynchronize(ctx->stream);
  }
  grx::release_device(ctx->dev);
  delete ctx;
  return GRXBLAS_STATUS_SUCCESS;
}

grxblasStatus_t grxblasSetStream(grxblasHandle_t handle, grxStream_t stream) {
  if (!handle) return GRXBLAS_STATUS_NOT_INITIALIZED;
  auto* ctx = reinterpret_cast<grxblasContext*>(handle);
  std::lock_guard<std::mutex> lock(ctx->mutex);
  ctx->stream = reinterpret_cast<cudaStream_t>(stream);
  return GRXBLAS_STATUS_SUCCESS;
}

grxblasStatus_t grxblasGetStream(grxblasHandle_t handle, grxStream_t* stream) {
  if (!handle || !stream) return GRXBLAS_STATUS_INVALID_VALUE;
  *stream = reinterpret_cast<grxStream_t>(reinterpret_cast<grxblasContext*>(handle)->stream);
  return GRXBLAS_STATUS_SUCCESS;
}

grxblasStatus_t grxblasSetKernelPath(const char* path) {
  std::lock_guard<std::mutex> lock(g_path_mutex);
  g_kernel_path = path ? path : "";
  return GRXBLAS_STATUS_SUCCESS;
}

grxblasStatus_t grxblasSetTensorMapSlots(grxblasHandle_t handle, int slotA, int slotB) {
  if (!handle) return GRXBLAS_STATUS_NOT_INITIALIZED;
  const int slots = 16;
  if (slotA < 0 || slotB < 0 || slotA >= slots || slotB >= slots || slotA == slotB)
    return GRXBLAS_STATUS_INVALID_VALUE;
  auto* ctx = reinterpret_cast<grxblasContext*>(handle);
  std::lock_guard<std::mutex> lock(ctx->mutex);
  ctx->slot_a = slotA;
  ctx->slot_b = slotB;
  return GRXBLAS_STATUS_SUCCESS;
}

grxblasStatus_t grxblasGetTensorTypes(grxblasHandle_t handle, unsigned* typeMask) {
  if (!handle) return GRXBLAS_STATUS_NOT_INITIALIZED;
  if (!typeMask) return GRXBLAS_STATUS_INVALID_VALUE;
  const grxblasStatus_t s = ensure(*reinterpret_cast<grxblasContext*>(handle), true);
  if (s != GRXBLAS_STATUS_SUCCESS) return s;
  *typeMask = GRXBLAS_TENSOR_FP16 | GRXBLAS_TENSOR_BF16 | GRXBLAS_TENSOR_FP8 | GRXBLAS_TENSOR_INT8;
  return GRXBLAS_STATUS_SUCCESS;
}

grxblasStatus_t grxblasGetTensorTile(grxblasHandle_t handle, int* m, int* n, int* k) {
  if (!handle) return GRXBLAS_STATUS_NOT_INITIALIZED;
  if (!m || !n || !k) return GRXBLAS_STATUS_INVALID_VALUE;
  const grxblasStatus_t s = ensure(*reinterpret_cast<grxblasContext*>(handle), true);
  if (s != GRXBLAS_STATUS_SUCCESS) return s;
  *m = grx::kTileM;
  *n = grx::kTileN;
  *k = 64;
  return GRXBLAS_STATUS_SUCCESS;
}

grxblasStatus_t grxblasGemmEx(grxblasHandle_t handle, grxblasOperation_t transa, grxblasOperation_t transb, int m,
                              int n, int k, const float* alpha, const void* A, grxDataType_t Atype, int lda,
                              const void* B, grxDataType_t Btype, int ldb, const float* beta, void* C,
                              grxDataType_t Ctype, int ldc) {
  return gemm_ex_impl(handle, transa, transb, m, n, k, alpha, A, Atype, lda, 0, B, Btype, ldb, 0, beta, C, Ctype,
                      ldc, 0, 1);
}

grxblasStatus_t grxblasGemmStridedBatchedEx(grxblasHandle_t handle, grxblasOperation_t transa,
                                            grxblasOperation_t transb, int m, int n, int k, const float* alpha,
                                            const void* A, grxDataType_t Atype, int lda, long long strideA,
                                            const void* B, grxDataType_t Btype, int ldb, long long strideB,
                                            const float* beta, void* C, grxDataType_t Ctype, int ldc,
                                            long long strideC, int batchCount) {
  return gemm_ex_impl(handle, transa, transb, m, n, k, alpha, A, Atype, lda, strideA, B, Btype, ldb, strideB, beta,
                      C, Ctype, ldc, strideC, batchCount);
}

grxblasStatus_t grxblasSetPeerOutputs(grxblasHandle_t handle, int n, void* const* peers) {
  if (!handle) return GRXBLAS_STATUS_NOT_INITIALIZED;
  if (n < 0 || n > grx::kMaxPeers || (n > 0 && !peers)) return GRXBLAS_STATUS_INVALID_VALUE;
  for (int i = 0; i < n; ++i)
    if (!peers[i]) return GRXBLAS_STATUS_INVALID_VALUE;
  auto* ctx = reinterpret_cast<grxblasContext*>(handle);
  std::lock_guard<std::mutex> lock(ctx->mutex);
  ctx->n_peers = peers ? n : 0;
  for (int i = 0; i < grx::kMaxPeers; ++i) ctx->peers[i] = i < ctx->n_peers ? peers[i] : nullptr;
  return GRXBLAS_STATUS_SUCCESS;
}

grxblasStatus_t grxblasSetEpilogue(grxblasHandle_t handle, const grxblasEpilogue_t* epilogue) {
  if (!handle) return GRXBLAS_STATUS_NOT_INITIALIZED;
  auto* ctx = reinterpret_cast<grxblasContext*>(handle);
  if (epilogue && ((unsigned)epilogue->scaleMode > 2u || (unsigned)epilogue->activation > 3u))
    return GRXBLAS_STATUS_INVALID_VALUE;
  std::lock_guard<std::mutex> lock(ctx->mutex);
  if (epilogue) {
    ctx->epi = *epilogue;
    ctx->has_epi = true;
  } else {
    ctx->epi = grxblasEpilogue_t{};
    ctx->has_epi = false;
  }
  return GRXBLAS_STATUS_SUCCESS;
}

grxblasStatus_t grxblasSetCycleProbe(grxblasHandle_t handle, grxCycleSlot* slots, int capacity) {
  if (!handle) return GRXBLAS_STATUS_NOT_INITIALIZED;
  if (slots && capacity <= 0) return GRXBLAS_STATUS_INVALID_VALUE;
  auto* ctx = reinterpret_cast<grxblasContext*>(handle);
  std::lock_guard<std::mutex> lock(ctx->mutex);
  ctx->probe = slots;
  ctx->probe_capacity = slots ? capacity : 0;
  return GRXBLAS_STATUS_SUCCESS;
}

// Slots for an m x n call of either kernel family: the sgemm grid (at batch 1,
// the smallest tile, so batch x this covers every batched call), or the
// tensor-core GEMM's persistent grid, which never exceeds the SM count nor two
// CTAs per 128 x 32 block of C.
int grxblasCycleSlotsNeeded(grxblasHandle_t handle, int m, int n) {
  (void)handle;
  if (m <= 0 || n <= 0) return 0;
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
    cudaGetLastError();
    sms = 148;  // no device: B200's count
  }
  const int sg = grx::sgemm_ctas(m, n, 1, sms);
  // tensor-core grid: at most one CTA per SM; with few tiles the single-CTA
  // kernel narrows them down to 32 columns (more CTAs)
  const long long tiles = 2LL * ((m + grx::kTileM - 1) / grx::kTileM) * ((n + 31) / 32);
  const int tc = (int)(tiles < sms ? tiles : sms);
  return sg > tc ? sg : tc;
}

grxblasStatus_t grxblasGetLoadedKernelPath(grxblasHandle_t handle, const char** path) {
  if (!handle) return GRXBLAS_STATUS_NOT_INITIALIZED;
  if (!path) return GRXBLAS_STATUS_INVALID_VALUE;
  auto* ctx = reinterpret_cast<grxblasContext*>(handle);
  std::lock_guard<std::mutex> lock(ctx->mutex);
  *path = ctx->loaded ? grx::library_path() : nullptr;
  return GRXBLAS_STATUS_SUCCESS;
}

grxblasStatus_t grxblasSetWorkspace(grxblasHandle_t handle, void* ws, size_t bytes) {
  if (!handle) return GRXBLAS_STATUS_NOT_INITIALIZED;
  if (ws && (reinterpret_cast<uintptr_t>(ws) & 255u)) return GRXBLAS_STATUS_INVALID_VALUE;
  auto* ctx = reinterpret_cast<grxblasContext*>(handle);
  std::lock_guard<std::mutex> lock(ctx->mutex);
  ctx->ws_user = ws;
  ctx->ws_user_bytes = ws ? bytes : 0;
  return GRXBLAS_STATUS_SUCCESS;
}

size_t grxblasGetWorkspaceSize(grxblasHandle_t handle, grxblasOperation_t transa, grxblasOperation_t transb, int m,
                               int n, int k, grxDataType_t Atype, int lda, grxDataType_t Btype, int ldb,
                               int batchCount) {
  (void)handle;
  (void)Btype;
  if (m <= 0 || n <= 0 || k <= 0 || batchCount <= 0) return 0;
  const int es = (Atype == GRX_R_16F || Atype == GRX_R_16BF) ? 2 : 1;
  // Upper bound: both operands packed, one copy per batch member (a call
  // whose operands are 16-byte aligned needs none of it), plus the split-K
  // scratch when the tile count leaves a partly idle last wave on this device.
  (void)transa;
  (void)transb;
  (void)lda;
  (void)ldb;
  const int kind = es == 2 ? grx::kKindF16 : (Atype == GRX_R_8I ? grx::kKindI8 : grx::kKindF8);
  size_t s = pack_bytes(m, k, es, batchCount) + pack_bytes(n, k, es, batchCount);
  s = (s + 255) & ~(size_t)255;
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) == cudaSuccess && cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess)
    s += grx::tc_gemm_splitk_bytes(kind, m, n, k, batchCount, sms);
  else
    cudaGetLastError();
  return s;
}

grxblasStatus_t grxblasGetExecutionStatus(grxblasHandle_t handle) {
  if (!handle) return GRXBLAS_STATUS_NOT_INITIALIZED;
  auto* ctx = reinterpret_cast<grxblasContext*>(handle);
  std::lock_guard<std::mutex> lock(ctx->mutex);
  const int code = grx::take_error(ctx->dev, ctx->stream);
  if (code < 0) return GRXBLAS_STATUS_EXECUTION_FAILED;
  return code == 0 ? GRXBLAS_STATUS_SUCCESS : GRXBLAS_STATUS_EXECUTION_FAILED;
}

// ------------------------------------------------------------ level 1 / 2

grxblasStatus_t grxblasSaxpy(grxblasHandle_t handle, int n, const float* alpha, const float* x, int incx, float* y,
                             int incy) {
  // reference grxblas.cpp:736-743
  if (!handle) return GRXBLAS_STATUS_NOT_INITIALIZED;
  if (!alpha) return GRXBLAS_STATUS_INVALID_VALUE;
  if (n < 0) return GRXBLAS_STATUS_INVALID_VALUE;
  if (n == 0) return GRXBLAS_STATUS_SUCCESS;
  if (!x || !y) return GRXBLAS_STATUS_INVALID_VALUE;
  if (incx == 0 || incy == 0) return GRXBLAS_STATUS_INVALID_VALUE;
  auto& ctx = *reinterpret_cast<grxblasContext*>(handle);
  const grxblasStatus_t s = ensure(ctx, false);
  if (s != GRXBLAS_STATUS_SUCCESS) return s;
  return from_cuda(grx::launch_saxpy(n, *alpha, x, incx, y, incy, ctx.stream));
}

grxblasStatus_t grxblasSscal(grxblasHandle_t handle, int n, const float* alpha, float* x, int incx) {
  // reference grxblas.cpp:777-785
  if (!handle) return GRXBLAS_STATUS_NOT_INITIALIZED;
  if (!alpha) return GRXBLAS_STATUS_INVALID_VALUE;
  if (n < 0) return GRXBLAS_STATUS_INVALID_VALUE;
  if (n == 0) return GRXBLAS_STATUS_SUCCESS;
  if (!x) return GRXBLAS_STATUS_INVALID_VALUE;
  if (incx <= 0) return GRXBLAS_STATUS_INVALID_VALUE;
  auto& ctx = *reinterpret_cast<grxblasContext*>(handle);
  const grxblasStatus_t s = ensure(ctx, false);
  if (s != GRXBLAS_STATUS_SUCCESS) return s;
  return from_cuda(grx::launch_sscal(n, *alpha, x, incx, ctx.stream));
}

grxblasStatus_t grxblasSgemv(grxblasHandle_t handle, grxblasOperation_t trans, int m, int n, const float* alpha,
                             const void* A, int lda, const void* x, int incx, const float* beta, void* y,
                             int incy) {
  // reference grxblas.cpp:815-827
  if (!handle) return GRXBLAS_STATUS_NOT_INITIALIZED;
  if (!alpha || !beta) return GRXBLAS_STATUS_INVALID_VALUE;
  if (m < 0 || n < 0) return GRXBLAS_STATUS_INVALID_VALUE;
  if (m == 0 || n == 0) return GRXBLAS_STATUS_SUCCESS;
  if (!A || !x || !y) return GRXBLAS_STATUS_INVALID_VALUE;
  if (incx == 0 || incy == 0) return GRXBLAS_STATUS_INVALID_VALUE;
  if (lda < m) return GRXBLAS_STATUS_INVALID_VALUE;
  auto& ctx = *reinterpret_cast<grxblasContext*>(handle);
  const grxblasStatus_t s = ensure(ctx, false);
  if (s != GRXBLAS_STATUS_SUCCESS) return s;
  return from_cuda(grx::launch_sgemv(trans == GRXBLAS_OP_T ? 1 : 0, m, n, *alpha, static_cast<const float*>(A), lda,
                                     static_cast<const float*>(x), incx, *beta, static_cast<float*>(y), incy,
                                     ctx.stream));
}

// ------------------------------------------------------------ SGEMM

static grxblasStatus_t sgemm_batched(grxblasHandle_t handle, grxblasOperation_t transa, grxblasOperation_t transb,
                                     int m, int n, int k, const float* alpha, const void* A, int lda,
                                     long long strideA, const void* B, int ldb, long long strideB,
                                     const float* beta, void* C, int ldc, long long strideC, int batch) {
  // reference grxblas.cpp:882-897
  if (!handle) return GRXBLAS_STATUS_NOT_INITIALIZED;
  if (!alpha || !beta) return GRXBLAS_STATUS_INVALID_VALUE;
  if (m < 0 || n < 0 || k < 0) return GRXBLAS_STATUS_INVALID_VALUE;
  if (batch < 0) return GRXBLAS_STATUS_INVALID_VALUE;
  if (m == 0 || n == 0 || batch == 0) return GRXBLAS_STATUS_SUCCESS;
  if (k > 0 && (!A || !B)) return GRXBLAS_STATUS_INVALID_VALUE;
  if (!C) return GRXBLAS_STATUS_INVALID_VALUE;
  const int min_lda = (transa == GRXBLAS_OP_N) ? m : k;
  const int min_ldb = (transb == GRXBLAS_OP_N) ? k : n;
  if (lda < min_lda || ldb < min_ldb || ldc < m) return GRXBLAS_STATUS_INVALID_VALUE;

  auto& ctx = *reinterpret_cast<grxblasContext*>(handle);
  std::lock_guard<std::mutex> lock(ctx.mutex);
  const grxblasStatus_t s = ensure_locked(ctx, false);
  if (s != GRXBLAS_STATUS_SUCCESS) return s;
  if (ctx.probe && ctx.probe_capacity < grx::sgemm_ctas(m, n, batch, ctx.dev.num_sms))
    return GRXBLAS_STATUS_INVALID_VALUE;

  grx::SgemmArgs a{};
  a.m = m;
  a.n = n;
  a.k = k;
  a.batch = batch;
  a.ta = transa == GRXBLAS_OP_T;
  a.tb = transb == GRXBLAS_OP_T;
  a.alpha = *alpha;
  a.beta = *beta;
  a.a = static_cast<const float*>(A);
  a.lda = lda;
  a.stride_a = strideA;
  a.b = static_cast<const float*>(B);
  a.ldb = ldb;
  a.stride_b = strideB;
  a.c = static_cast<float*>(C);
  a.ldc = ldc;
  a.stride_c = strideC;
  a.probe = ctx.probe;
  return from_cuda(grx::launch_sgemm(a, ctx.dev.num_sms, ctx.stream));
}

grxblasStatus_t grxblasSgemm(grxblasHandle_t handle, grxblasOperation_t transa, grxblasOperation_t transb, int m,
                             int n, int k, const float* alpha, const void* A, int lda, const void* B, int ldb,
                             const float* beta, void* C, int ldc) {
  return sgemm_batched(handle, transa, transb, m, n, k, alpha, A, lda, 0, B, ldb, 0, beta, C, ldc, 0, 1);
}

grxblasStatus_t grxblasSgemmStridedBatched(grxblasHandle_t handle, grxblasOperation_t transa,
                                           grxblasOperation_t transb, int m, int n, int k, const float* alpha,
                                           const void* A, int lda, long long strideA, const void* B, int ldb,
                                           long long strideB, const float* beta, void* C, int ldc,
                                           long long strideC, int batchCount) {
  return sgemm_batched(handle, transa, transb, m, n, k, alpha, A, lda, strideA, B, ldb, strideB, beta, C, ldc,
                       strideC, batchCount);
}

}  // extern "C"
