/* grxcp-b200 -- grxBLAS: dense linear algebra on B200 (sm_100a).
 *
 * Drop-in for the reference's grxBLAS C API (include/grx/grxblas.h of
 * kubeworkz/grxcp): every prototype below that carries a "reference" citation
 * has the reference's exact signature, argument meaning, status codes and
 * refusal rules. Entry points marked "additive" do not exist in the reference;
 * they extend it for types and fusions the B200 tensor cores provide.
 *
 * Conventions (unchanged from the reference):
 *   column-major storage, C = alpha * op(A) * op(B) + beta * C
 *   A is m x k (stored k x m when transposed), B is k x n, C is m x n
 *   element (i, j) of a stored matrix with leading dimension ld is at [i + j*ld]
 *   all matrix pointers are device addresses; alpha/beta are HOST pointers
 *   beta == 0 never reads C (C may hold NaN or garbage)
 *   every call is enqueued on the handle's stream and returns without a host
 *   synchronisation
 */
#ifndef GRXBLAS_H
#define GRXBLAS_H

#include "grx_cycles.h"
#include "grx_runtime.h"
#include "grx_tensormap.h"
#include "grx_types.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct grxblasContext* grxblasHandle_t;

/* reference grxblas.h:37-46 */
typedef enum {
  GRXBLAS_STATUS_SUCCESS          = 0,
  GRXBLAS_STATUS_NOT_INITIALIZED  = 1,
  GRXBLAS_STATUS_ALLOC_FAILED     = 2,
  GRXBLAS_STATUS_INVALID_VALUE    = 3,
  GRXBLAS_STATUS_ARCH_MISMATCH    = 4,
  GRXBLAS_STATUS_EXECUTION_FAILED = 5,
  GRXBLAS_STATUS_NOT_SUPPORTED    = 6,
  GRXBLAS_STATUS_INTERNAL_ERROR   = 7
} grxblasStatus_t;

/* reference grxblas.h:48-51 */
typedef enum {
  GRXBLAS_OP_N = 0,
  GRXBLAS_OP_T = 1
} grxblasOperation_t;

/* reference grxblas.h:119-126; GRXBLAS_TENSOR_BF16 is additive. */
typedef enum {
  GRXBLAS_TENSOR_FP16 = 0x01,
  GRXBLAS_TENSOR_TF32 = 0x02,
  GRXBLAS_TENSOR_FP8  = 0x04,
  GRXBLAS_TENSOR_FP4  = 0x08,
  GRXBLAS_TENSOR_INT8 = 0x10,
  GRXBLAS_TENSOR_INT4 = 0x20,
  GRXBLAS_TENSOR_BF16 = 0x40
} grxblasTensorType_t;

/* reference grxblas.h:53, grxblas.cpp:412-424 */
const char* grxblasGetStatusString(grxblasStatus_t s);

/* reference grxblas.h:55-58, grxblas.cpp:426-450 */
grxblasStatus_t grxblasCreate(grxblasHandle_t* handle);
grxblasStatus_t grxblasDestroy(grxblasHandle_t handle);
grxblasStatus_t grxblasSetStream(grxblasHandle_t handle, grxStream_t stream);
grxblasStatus_t grxblasGetStream(grxblasHandle_t handle, grxStream_t* stream);

/* Tensor-core GEMM. reference grxblas.h:97-105, grxblas.cpp:498-702.
 *
 * Accepted type triples (Atype, Btype, Ctype):
 *   16F,  16F,  32F    reference pairing: fp16 in, fp32 accumulate and out
 *   16F,  16F,  16F    additive
 *   16BF, 16BF, 32F    additive
 *   16BF, 16BF, 16BF   additive
 *   8I,   8I,   32I    reference pairing: int8 in, int32 accumulate and out,
 *                      alpha/beta must hold exact integers, bit-exact result
 *   8I,   8I,   16BF   additive, needs a per-row/per-column scale epilogue
 *   8F_E4M3, 8F_E4M3, 16BF or 32F   additive, per-tensor scale epilogue
 * Anything else returns NOT_SUPPORTED (one explanatory stderr line per
 * process); nothing falls back to a slower kernel. The epilogue installed with
 * grxblasSetEpilogue (bias, scales) applies to this call. */
grxblasStatus_t grxblasGemmEx(grxblasHandle_t handle,
                              grxblasOperation_t transa,
                              grxblasOperation_t transb,
                              int m, int n, int k,
                              const float* alpha,
                              const void* A, grxDataType_t Atype, int lda,
                              const void* B, grxDataType_t Btype, int ldb,
                              const float* beta,
                              void* C, grxDataType_t Ctype, int ldc);

/* Additive: GemmEx over a batch at constant element strides (signed; 0
 * broadcasts an operand, as grxblasSgemmStridedBatched allows). One launch for
 * the whole batch. batchCount < 0 is INVALID_VALUE, 0 is SUCCESS. */
grxblasStatus_t grxblasGemmStridedBatchedEx(
    grxblasHandle_t handle, grxblasOperation_t transa, grxblasOperation_t transb,
    int m, int n, int k, const float* alpha,
    const void* A, grxDataType_t Atype, int lda, long long strideA,
    const void* B, grxDataType_t Btype, int ldb, long long strideB,
    const float* beta,
    void* C, grxDataType_t Ctype, int ldc, long long strideC, int batchCount);

/* Additive: fused epilogue of the tensor-core GEMM.
 *
 *   D(i,j) = act( alpha * s(i,j) * acc(i,j) + beta * C(i,j) + bias[j or i] )
 *
 * with s(i,j) = 1 (NONE), scaleA[0]*scaleB[0] (TENSOR), or scaleA[i]*scaleB[j]
 * (ROWCOL: i over the m rows of op(A), j over the n columns of op(B)). bias,
 * scaleA and scaleB are DEVICE pointers (so quantisation scales computed on
 * the GPU need no round trip); bias may be NULL. Batch strides are in elements
 * and apply per batch member of a strided-batched call. The epilogue is
 * copied into the handle and applies to every later GemmEx call on it until
 * replaced; NULL restores the plain alpha/beta epilogue. The int32-out int8
 * pairing accepts only the plain epilogue (its result is exact by contract).
 * biasOverRows = 0 indexes the bias by column j (length n), 1 by row i (length
 * m: the per-output-feature bias of a linear layer computed as C = W^T X with
 * row-major activations). activation is applied last (GELU per the erf
 * definition or its tanh approximation). */
typedef enum {
  GRXBLAS_SCALE_NONE   = 0,
  GRXBLAS_SCALE_TENSOR = 1,
  GRXBLAS_SCALE_ROWCOL = 2
} grxblasScaleMode_t;

typedef enum {
  GRXBLAS_ACT_NONE      = 0,
  GRXBLAS_ACT_RELU      = 1,
  GRXBLAS_ACT_GELU_TANH = 2,
  GRXBLAS_ACT_GELU_ERF  = 3
} grxblasActivation_t;

typedef struct {
  const void*        bias;        /* [n] (or [m], see biasOverRows) per batch member, or NULL */
  grxDataType_t      biasType;    /* GRX_R_32F or GRX_R_16BF */
  long long          strideBias;
  grxblasScaleMode_t scaleMode;
  const float*       scaleA;      /* [1] or [m] */
  const float*       scaleB;      /* [1] or [n] */
  long long          strideScaleA;
  long long          strideScaleB;
  int                biasOverRows;
  grxblasActivation_t activation;
} grxblasEpilogue_t;

grxblasStatus_t grxblasSetEpilogue(grxblasHandle_t handle, const grxblasEpilogue_t* epilogue);

/* Replicated output (no counterpart in the reference, which has no
 * multi-device path). After this call, every element a 16-bit GemmEx /
 * GemmStridedBatchedEx on this handle stores to C is also stored at the same
 * element offset in each of the n peer buffers -- other GPUs' copies of C,
 * opened in this process with grxIpcOpenMemHandle -- from the same kernel's
 * epilogue, over NVLink. With one process per GPU each computing its own
 * columns of C, this assembles C on every GPU in the GEMM itself, without a
 * separate all-gather. The caller must order the peers' reads after every
 * writer's kernel (for example a cross-rank barrier). n <= 7; n == 0 or
 * peers == NULL clears. GemmEx with peers set and k == 0, or with 8-bit
 * inputs, returns NOT_SUPPORTED. */
grxblasStatus_t grxblasSetPeerOutputs(grxblasHandle_t handle, int n, void* const* peers);

/* reference grxblas.h:131-132. Reports FP16|BF16|FP8|INT8 on B200. */
grxblasStatus_t grxblasGetTensorTypes(grxblasHandle_t handle, unsigned* typeMask);

/* reference grxblas.h:135-136. Operand descriptors are TMA tensor maps built per
 * launch and passed as kernel parameters, so there is no device descriptor
 * state to collide with; the slots are validated (0 <= slot < 16, distinct)
 * and recorded, nothing more. */
grxblasStatus_t grxblasSetTensorMapSlots(grxblasHandle_t handle, int slotA, int slotB);

/* reference grxblas.h:143-144. The CTA tile GemmEx blocks a 16-bit problem
 * into: 128 x 256 outputs per tile, 64 of k per pipeline stage. */
grxblasStatus_t grxblasGetTensorTile(grxblasHandle_t handle, int* m, int* n, int* k);

/* Level 1 / level 2 (reference grxblas.h:161-181). Increments follow BLAS,
 * negative walks backwards, zero is refused; sscal needs incx > 0. */
grxblasStatus_t grxblasSaxpy(grxblasHandle_t handle, int n, const float* alpha,
                             const float* x, int incx, float* y, int incy);
grxblasStatus_t grxblasSscal(grxblasHandle_t handle, int n, const float* alpha,
                             float* x, int incx);
grxblasStatus_t grxblasSgemv(grxblasHandle_t handle, grxblasOperation_t trans,
                             int m, int n, const float* alpha,
                             const void* A, int lda,
                             const void* x, int incx,
                             const float* beta,
                             void* y, int incy);

/* fp32 GEMM on the FP32 pipe (no TF32). reference grxblas.h:187-195. */
grxblasStatus_t grxblasSgemm(grxblasHandle_t handle,
                             grxblasOperation_t transa,
                             grxblasOperation_t transb,
                             int m, int n, int k,
                             const float* alpha,
                             const void* A, int lda,
                             const void* B, int ldb,
                             const float* beta,
                             void* C, int ldc);

/* reference grxblas.h:207-212 */
grxblasStatus_t grxblasSgemmStridedBatched(
    grxblasHandle_t handle, grxblasOperation_t transa,
    grxblasOperation_t transb, int m, int n, int k, const float* alpha,
    const void* A, int lda, long long strideA,
    const void* B, int ldb, long long strideB,
    const float* beta, void* C, int ldc, long long strideC, int batchCount);

/* reference grxblas.h:227. The kernels are compiled into this library, so a
 * configured path must name this library file or its directory; any other
 * configured path makes later calls return NOT_INITIALIZED (no fallback past a
 * configured path, as in the reference). NULL or "" clears it. */
grxblasStatus_t grxblasSetKernelPath(const char* path);

/* reference grxblas.h:240-242. `slots` is a DEVICE array; the next sgemm writes
 * one grxCycleSlot per CTA. */
grxblasStatus_t grxblasSetCycleProbe(grxblasHandle_t handle, grxCycleSlot* slots, int capacity);
int             grxblasCycleSlotsNeeded(grxblasHandle_t handle, int m, int n);

/* reference grxblas.h:247-248. The file the kernels run from (this library). */
grxblasStatus_t grxblasGetLoadedKernelPath(grxblasHandle_t handle, const char** path);

/* Additive: caller-provided scratch for the operand-packing path (used when an
 * operand's address or leading dimension is not 16-byte aligned, or an
 * operand stride is negative). Without it the handle allocates its own on first
 * need. grxblasGetWorkspaceSize reports the bytes a call would need. */
grxblasStatus_t grxblasSetWorkspace(grxblasHandle_t handle, void* workspace, size_t bytes);
size_t          grxblasGetWorkspaceSize(grxblasHandle_t handle, grxblasOperation_t transa,
                                        grxblasOperation_t transb, int m, int n, int k,
                                        grxDataType_t Atype, int lda, grxDataType_t Btype,
                                        int ldb, int batchCount);

/* Additive: synchronises the handle's stream and reports whether any kernel
 * launched through this handle gave up on a bounded wait since the last query
 * (EXECUTION_FAILED), or whether the stream reported an error. Clears the flag. */
grxblasStatus_t grxblasGetExecutionStatus(grxblasHandle_t handle);

/* Additive (no counterpart in the reference, which runs on one device):
 * column-parallel GemmEx across GPUs, one process per GPU, over NCCL.
 *
 *   rank 0:       grxblasShardGetUniqueId(&id); send id to the other ranks
 *   every rank:   grxblasShardCommInit(&comm, &id, rank, world)   (current device)
 *                 grxblasGemmExColumnParallel(handle, comm, ..., replicate)
 *                 grxblasShardSynchronize(handle, comm)
 *                 grxblasShardCommDestroy(comm)
 *
 * grxblasGemmExColumnParallel takes the arguments of grxblasGemmEx for the
 * WHOLE problem (B and C are the full n-column operands; A is replicated) and
 * computes this rank's columns grxblasShardRange(n, rank, world) with one local
 * GemmEx on the handle's stream; the handle's epilogue applies, with per-column
 * bias and scales read at the same global columns. replicate != 0 then
 * broadcasts every rank's column block of C (its ld padding rows included) so
 * that C is complete on every rank; replicate == 0 leaves each rank its own
 * columns only. Calls return after enqueueing; every rank must make the same
 * calls in the same order.
 *
 * Failures are detected on the host: the communicator is non-blocking, and
 * initialisation, each enqueue and grxblasShardSynchronize give up after
 * GRX_SHARD_TIMEOUT_MS (default 60000 ms; a rank that never joined or has
 * left), abort the communicator and return EXECUTION_FAILED. An aborted
 * communicator refuses further calls with EXECUTION_FAILED and must be
 * destroyed. NOT_SUPPORTED: libnccl.so.2 could not be loaded. */
typedef struct {
  char internal[128];
} grxblasShardUniqueId_t;
typedef struct grxblasShardContext* grxblasShardComm_t;

grxblasStatus_t grxblasShardGetUniqueId(grxblasShardUniqueId_t* id);
grxblasStatus_t grxblasShardCommInit(grxblasShardComm_t* comm, const grxblasShardUniqueId_t* id,
                                     int rank, int world);
grxblasStatus_t grxblasShardCommDestroy(grxblasShardComm_t comm);
/* Contiguous split of n columns: the first n % world ranks get one more. */
grxblasStatus_t grxblasShardRange(int n, int rank, int world, int* start, int* count);
grxblasStatus_t grxblasGemmExColumnParallel(grxblasHandle_t handle, grxblasShardComm_t comm,
                                            grxblasOperation_t transa, grxblasOperation_t transb,
                                            int m, int n, int k, const float* alpha,
                                            const void* A, grxDataType_t Atype, int lda,
                                            const void* B, grxDataType_t Btype, int ldb,
                                            const float* beta,
                                            void* C, grxDataType_t Ctype, int ldc, int replicate);
/* Waits (bounded, as above) for the handle's stream, including the broadcasts,
 * then reports grxblasGetExecutionStatus. */
grxblasStatus_t grxblasShardSynchronize(grxblasHandle_t handle, grxblasShardComm_t comm);

/* No counterpart in the reference. grxblasGemmEx for callers that may not
 * allocate device memory -- code whose device memory is owned by another
 * allocator (framework plug-ins, fixed-budget serving processes) or that must
 * not trigger cudaMalloc's implicit synchronisation. Same arguments and type
 * pairings as grxblasGemmEx, without a handle (plain alpha/beta epilogue, no
 * bias or scales), enqueued on `stream`. It allocates nothing: operands that
 * must be packed (address or leading dimension not 16-byte aligned) go to a
 * fixed 16 MiB device array inside this library, which every GPU that loads the
 * library holds until exit; a problem needing more packing scratch than that
 * is refused with INVALID_VALUE and a stderr line. `errorFlag` is an optional
 * device int the kernel sets non-zero if it gives up on a bounded wait. The
 * first call on each device resolves the array's device address (make it
 * before any stream capture). All calls share the array: calls that overlap on
 * the GPU race and must be ordered by the caller. */
grxblasStatus_t grxblasGemmExNoAlloc(grxStream_t stream,
                                     grxblasOperation_t transa,
                                     grxblasOperation_t transb,
                                     int m, int n, int k,
                                     const float* alpha,
                                     const void* A, grxDataType_t Atype, int lda,
                                     const void* B, grxDataType_t Btype, int ldb,
                                     const float* beta,
                                     void* C, grxDataType_t Ctype, int ldc,
                                     int* errorFlag);

#ifdef __cplusplus
}
#endif

#endif /* GRXBLAS_H */
