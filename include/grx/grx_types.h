/* grxcp-b200 -- core types of the host runtime boundary.
 *
 * Binary-compatible with the GRXCP core types header (include/grx/grx_types.h
 * in kubeworkz/grxcp): the same enumerator values, the same struct field order,
 * so code compiled against the reference headers links against this library
 * unchanged. Two element types are added (bf16 and fp8 e4m3) with the values
 * CUDA's cudaDataType uses for them, which is the numbering the reference
 * already follows for the types it has.
 *
 * On B200 a grxStream_t IS a cudaStream_t (the pointer value is passed through
 * unchanged), and a grxEvent_t IS a cudaEvent_t. Device pointers are CUDA
 * device pointers.
 */
#ifndef GRX_TYPES_H
#define GRX_TYPES_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Errors. Values follow grx_types.h:22-45 of the reference. */
typedef enum {
  grxSuccess                     = 0,
  grxErrorInvalidValue           = 1,
  grxErrorMemoryAllocation       = 2,
  grxErrorInitializationError    = 3,
  grxErrorInvalidDevice          = 4,
  grxErrorInvalidDevicePointer   = 5,
  grxErrorInvalidMemcpyDirection = 6,
  grxErrorInvalidResourceHandle  = 7,
  grxErrorNotReady               = 8,
  grxErrorNotSupported           = 9,
  grxErrorInvalidKernelImage     = 10,
  grxErrorInvalidDeviceFunction  = 11,
  grxErrorLaunchFailure          = 12,
  grxErrorLaunchOutOfResources   = 13,
  grxErrorDeviceLost             = 14,
  grxErrorTimeout                = 15,
  grxErrorFileNotFound           = 16,
  grxErrorInvalidSymbol          = 17,
  grxErrorUnknown                = 999
} grxError_t;

const char* grxGetErrorName(grxError_t e);
const char* grxGetErrorString(grxError_t e);

typedef struct { unsigned int x, y, z; } dim3_t;

/* Opaque handles. On this implementation they carry CUDA handles verbatim. */
typedef struct grxStream* grxStream_t;
typedef struct grxEvent*  grxEvent_t;

#define grxStreamDefault      0x00u
#define grxStreamNonBlocking  0x01u
#define grxEventDefault       0x00u
#define grxEventBlockingSync  0x01u
#define grxEventDisableTiming 0x02u

typedef enum {
  grxMemcpyHostToHost     = 0,
  grxMemcpyHostToDevice   = 1,
  grxMemcpyDeviceToHost   = 2,
  grxMemcpyDeviceToDevice = 3,
  grxMemcpyDefault        = 4   /* direction inferred from the pointers (UVA) */
} grxMemcpyKind;

/* Element types. GRX_R_16F/32F/8I/32I are the reference's (grx_types.h:120-134);
 * GRX_R_16BF and GRX_R_8F_E4M3 are additive, numbered as CUDA_R_16BF and
 * CUDA_R_8F_E4M3. */
typedef enum {
  GRX_R_32F     = 0,
  GRX_R_16F     = 2,
  GRX_R_8I      = 3,
  GRX_R_32I     = 10,
  GRX_R_16BF    = 14,
  GRX_R_8F_E4M3 = 28
} grxDataType_t;

typedef enum { GRX_DEVICE_TYPE_GPU = 0, GRX_DEVICE_TYPE_NPU = 1 } grxDeviceType_t;

typedef enum {
  GRX_BACKEND_SIMX    = 0,
  GRX_BACKEND_RTLSIM  = 1,
  GRX_BACKEND_XRT     = 2,
  GRX_BACKEND_OPAE    = 3,
  GRX_BACKEND_GEM5    = 4,
  GRX_BACKEND_SILICON = 5
} grxBackend_t;

#define GRX_CAP_KERNEL_LAUNCH      (1u << 0)
#define GRX_CAP_STREAMS            (1u << 1)
#define GRX_CAP_EVENTS             (1u << 2)
#define GRX_CAP_MEMCPY             (1u << 3)
#define GRX_CAP_GEMM               (1u << 4)
#define GRX_CAP_UNIFIED_ADDRESSING (1u << 5)
#define GRX_CAP_TENSOR_CORE        (1u << 6)
#define GRX_CAP_ASYNC_COPY         (1u << 7)
#define GRX_CAP_RAY_TRACING        (1u << 8)
#define GRX_CAP_COOPERATIVE_LAUNCH (1u << 9)
#define GRX_CAP_GLOBAL_ATOMICS     (1u << 10)

/* Device description. Field order is the reference's (grx_types.h:176-216) so
 * the struct is ABI-identical; on B200 every field is filled from
 * cudaGetDeviceProperties. */
typedef struct {
  char            name[128];
  grxDeviceType_t deviceType;
  grxBackend_t    backend;
  unsigned int    capabilities;
  int             computeCapabilityMajor;
  int             computeCapabilityMinor;
  int    warpSize;
  int    maxWarpsPerMultiProcessor;
  int    multiProcessorCount;
  int    clusterCount;
  int    socketSize;
  int    issueWidth;
  int    maxThreadsPerBlock;
  int    maxThreadsDim[3];
  int    maxGridSize[3];
  int    numBarriers;
  size_t totalGlobalMem;
  size_t sharedMemPerMultiprocessor;
  size_t sharedMemPerBlock;
  int    memBankCount;
  size_t memBankSize;
  int    cacheLineSize;
  int    clockRateMHz;
  size_t peakMemoryBandwidthMBs;
  int    unifiedAddressing;
  int    managedMemory;
  size_t pinnedMemTotal;
  size_t pinnedMemFree;
  int    warpShuffleIsEmulated;
  int    eventTimingIsDeviceSide;
  int    constantMemoryIsGlobal;
} grxDeviceProp_t;

#ifdef __cplusplus
}
#endif

#endif /* GRX_TYPES_H */
