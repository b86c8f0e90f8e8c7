/* grxcp-b200 -- the subset of the GRXCP host runtime (libgrxrt) that grxBLAS
 * and grxDNN callers use, implemented over the CUDA runtime.
 *
 * Every prototype here is the reference's (include/grx/grx_runtime.h:25-150 in
 * kubeworkz/grxcp); semantics are CUDA's, as they are in the reference. Entry
 * points of the reference runtime that only concern its own device toolchain
 * (module loading, fatbin registration, descriptor slots, occupancy for the
 * G100 dispatcher) are not part of this library.
 */
#ifndef GRX_RUNTIME_H
#define GRX_RUNTIME_H

#include "grx_types.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Device management -- reference grx_runtime.h:25-32 */
grxError_t grxGetDeviceCount(int* count);
grxError_t grxSetDevice(int device);
grxError_t grxGetDevice(int* device);
grxError_t grxGetDeviceProperties(grxDeviceProp_t* prop, int device);
grxError_t grxDeviceSynchronize(void);
grxError_t grxMemGetInfo(size_t* freeBytes, size_t* totalBytes);

/* Peer access -- reference grx_runtime.h:37-38. The reference refuses; on an
 * NVSwitch box every peer is reachable, so these answer truthfully. */
grxError_t grxDeviceCanAccessPeer(int* canAccess, int device, int peer);
grxError_t grxDeviceEnablePeerAccess(int peerDevice, unsigned int flags);

/* Inter-process device memory (no counterpart in the reference): export a
 * handle to a grxMalloc allocation, open a peer process's handle as a device
 * pointer of this process (peer access enabled lazily), close it. One process
 * per GPU uses these to let kernels store straight into a peer's buffer over
 * NVLink (grxblasSetPeerOutputs). devPtr must be the base of an allocation. */
typedef struct {
  unsigned char reserved[64];
} grxIpcMemHandle_t;
grxError_t grxIpcGetMemHandle(grxIpcMemHandle_t* handle, void* devPtr);
grxError_t grxIpcOpenMemHandle(void** devPtr, grxIpcMemHandle_t handle);
grxError_t grxIpcCloseMemHandle(void* devPtr);

/* Sticky last error -- reference grx_runtime.h:44-45 */
grxError_t grxGetLastError(void);
grxError_t grxPeekAtLastError(void);

/* Memory -- reference grx_runtime.h:51-77 */
grxError_t grxMalloc(void** ptr, size_t size);
grxError_t grxFree(void* ptr);
grxError_t grxMallocHost(void** ptr, size_t size);
grxError_t grxFreeHost(void* ptr);
grxError_t grxMemcpy(void* dst, const void* src, size_t count, grxMemcpyKind kind);
grxError_t grxMemcpyAsync(void* dst, const void* src, size_t count,
                          grxMemcpyKind kind, grxStream_t stream);
grxError_t grxMemset(void* dst, int value, size_t count);
grxError_t grxMemsetAsync(void* dst, int value, size_t count, grxStream_t stream);

/* Streams -- reference grx_runtime.h:90-97 */
grxError_t grxStreamCreate(grxStream_t* stream);
grxError_t grxStreamCreateWithFlags(grxStream_t* stream, unsigned int flags);
grxError_t grxStreamDestroy(grxStream_t stream);
grxError_t grxStreamSynchronize(grxStream_t stream);
grxError_t grxStreamQuery(grxStream_t stream);
grxError_t grxStreamWaitEvent(grxStream_t stream, grxEvent_t event, unsigned int flags);

/* Events -- reference grx_runtime.h:110-116. Timing is device-side (CUDA
 * events), so grxDeviceProp_t.eventTimingIsDeviceSide is 1. */
grxError_t grxEventCreate(grxEvent_t* event);
grxError_t grxEventCreateWithFlags(grxEvent_t* event, unsigned int flags);
grxError_t grxEventDestroy(grxEvent_t event);
grxError_t grxEventRecord(grxEvent_t event, grxStream_t stream);
grxError_t grxEventSynchronize(grxEvent_t event);
grxError_t grxEventQuery(grxEvent_t event);
grxError_t grxEventElapsedTime(float* ms, grxEvent_t start, grxEvent_t end);

#ifdef __cplusplus
}
#endif

#endif /* GRX_RUNTIME_H */
