// libgrxrt subset over the CUDA runtime.
//
// The reference runtime (src/runtime/*.cpp) drives a GRX-G100 through the
// vortex2.h driver; here every entry point maps onto its CUDA analogue. The
// sticky last-error semantics follow src/runtime/error.cpp:30-48: every call
// that fails records its error for grxGetLastError (returns and clears) and
// grxPeekAtLastError (returns).
#include <cuda_runtime.h>
#include <string.h>

#include "grx/grx_runtime.h"
#include "grx/grx_tensormap.h"

namespace {

thread_local grxError_t g_last_error = grxSuccess;

grxError_t map_cuda(cudaError_t e) {
  switch (e) {
    case cudaSuccess: return grxSuccess;
    case cudaErrorInvalidValue: return grxErrorInvalidValue;
    case cudaErrorMemoryAllocation: return grxErrorMemoryAllocation;
    case cudaErrorInitializationError:
    case cudaErrorInsufficientDriver:
    case cudaErrorNoDevice: return grxErrorInitializationError;
    case cudaErrorInvalidDevice: return grxErrorInvalidDevice;
    case cudaErrorInvalidDevicePointer: return grxErrorInvalidDevicePointer;
    case cudaErrorInvalidMemcpyDirection: return grxErrorInvalidMemcpyDirection;
    case cudaErrorInvalidResourceHandle: return grxErrorInvalidResourceHandle;
    case cudaErrorNotReady: return grxErrorNotReady;
    case cudaErrorNotSupported: return grxErrorNotSupported;
    case cudaErrorInvalidKernelImage:
    case cudaErrorNoKernelImageForDevice: return grxErrorInvalidKernelImage;
    case cudaErrorInvalidDeviceFunction: return grxErrorInvalidDeviceFunction;
    case cudaErrorLaunchFailure: return grxErrorLaunchFailure;
    case cudaErrorLaunchOutOfResources: return grxErrorLaunchOutOfResources;
    case cudaErrorLaunchTimeout: return grxErrorTimeout;
    case cudaErrorInvalidSymbol: return grxErrorInvalidSymbol;
    case cudaErrorFileNotFound: return grxErrorFileNotFound;
    default: return grxErrorUnknown;
  }
}

grxError_t rec(cudaError_t e) {
  const grxError_t g = map_cuda(e);
  if (g != grxSuccess) g_last_error = g;
  return g;
}

grxError_t rec_g(grxError_t g) {
  if (g != grxSuccess) g_last_error = g;
  return g;
}

cudaStream_t cs(grxStream_t s) { return reinterpret_cast<cudaStream_t>(s); }
cudaEvent_t ce(grxEvent_t e) { return reinterpret_cast<cudaEvent_t>(e); }

}  // namespace

extern "C" {

const char* grxGetErrorName(grxError_t e) {
  switch (e) {
    case grxSuccess: return "grxSuccess";
    case grxErrorInvalidValue: return "grxErrorInvalidValue";
    case grxErrorMemoryAllocation: return "grxErrorMemoryAllocation";
    case grxErrorInitializationError: return "grxErrorInitializationError";
    case grxErrorInvalidDevice: return "grxErrorInvalidDevice";
    case grxErrorInvalidDevicePointer: return "grxErrorInvalidDevicePointer";
    case grxErrorInvalidMemcpyDirection: return "grxErrorInvalidMemcpyDirection";
    case grxErrorInvalidResourceHandle: return "grxErrorInvalidResourceHandle";
    case grxErrorNotReady: return "grxErrorNotReady";
    case grxErrorNotSupported: return "grxErrorNotSupported";
    case grxErrorInvalidKernelImage: return "grxErrorInvalidKernelImage";
    case grxErrorInvalidDeviceFunction: return "grxErrorInvalidDeviceFunction";
    case grxErrorLaunchFailure: return "grxErrorLaunchFailure";
    case grxErrorLaunchOutOfResources: return "grxErrorLaunchOutOfResources";
    case grxErrorDeviceLost: return "grxErrorDeviceLost";
    case grxErrorTimeout: return "grxErrorTimeout";
    case grxErrorFileNotFound: return "grxErrorFileNotFound";
    case grxErrorInvalidSymbol: return "grxErrorInvalidSymbol";
    case grxErrorUnknown: return "grxErrorUnknown";
  }
  return "grxErrorUnknown";
}

const char* grxGetErrorString(grxError_t e) {
  switch (e) {
    case grxSuccess: return "no error";
    case grxErrorInvalidValue: return "invalid argument";
    case grxErrorMemoryAllocation: return "out of memory";
    case grxErrorInitializationError: return "initialization error (no usable CUDA device or driver)";
    case grxErrorInvalidDevice: return "invalid device ordinal";
    case grxErrorInvalidDevicePointer: return "invalid device pointer";
    case grxErrorInvalidMemcpyDirection: return "invalid copy direction";
    case grxErrorInvalidResourceHandle: return "invalid resource handle";
    case grxErrorNotReady: return "device not ready";
    case grxErrorNotSupported: return "operation not supported";
    case grxErrorInvalidKernelImage: return "no kernel image for this device";
    case grxErrorInvalidDeviceFunction: return "invalid device function";
    case grxErrorLaunchFailure: return "launch failure";
    case grxErrorLaunchOutOfResources: return "too many resources requested for launch";
    case grxErrorDeviceLost: return "device lost";
    case grxErrorTimeout: return "timeout";
    case grxErrorFileNotFound: return "file not found";
    case grxErrorInvalidSymbol: return "invalid device symbol";
    case grxErrorUnknown: return "unknown error";
  }
  return "unknown error";
}

grxError_t grxGetDeviceCount(int* count) {
  if (!count) return rec_g(grxErrorInvalidValue);
  int c = 0;
  const cudaError_t e = cudaGetDeviceCount(&c);
  if (e == cudaErrorNoDevice || e == cudaErrorInsufficientDriver) {
    cudaGetLastError();
    *count = 0;
    return grxSuccess;
  }
  *count = c;
  return rec(e);
}

grxError_t grxSetDevice(int device) { return rec(cudaSetDevice(device)); }
grxError_t grxGetDevice(int* device) { return device ? rec(cudaGetDevice(device)) : rec_g(grxErrorInvalidValue); }

grxError_t grxGetDeviceProperties(grxDeviceProp_t* prop, int device) {
  if (!prop) return rec_g(grxErrorInvalidValue);
  cudaDeviceProp p;
  const cudaError_t e = cudaGetDeviceProperties(&p, device);
  if (e != cudaSuccess) return rec(e);
  memset(prop, 0, sizeof(*prop));
  strncpy(prop->name, p.name, sizeof(prop->name) - 1);
  prop->deviceType = GRX_DEVICE_TYPE_GPU;
  prop->backend = GRX_BACKEND_SILICON;
  unsigned caps = GRX_CAP_KERNEL_LAUNCH | GRX_CAP_STREAMS | GRX_CAP_EVENTS | GRX_CAP_MEMCPY | GRX_CAP_GEMM |
                  GRX_CAP_UNIFIED_ADDRESSING | GRX_CAP_GLOBAL_ATOMICS | GRX_CAP_COOPERATIVE_LAUNCH;
  // The tcgen05 tensor cores and the TMA engine are sm_100 features.
  if (p.major == 10) caps |= GRX_CAP_TENSOR_CORE | GRX_CAP_ASYNC_COPY;
  prop->capabilities = caps;
  prop->computeCapabilityMajor = p.major;
  prop->computeCapabilityMinor = p.minor;
  prop->warpSize = p.warpSize;
  prop->maxWarpsPerMultiProcessor = p.maxThreadsPerMultiProcessor / p.warpSize;
  prop->multiProcessorCount = p.multiProcessorCount;
  prop->clusterCount = 1;
  prop->socketSize = 1;
  prop->issueWidth = 4;
  prop->maxThreadsPerBlock = p.maxThreadsPerBlock;
  for (int i = 0; i < 3; ++i) {
    prop->maxThreadsDim[i] = p.maxThreadsDim[i];
    prop->maxGridSize[i] = p.maxGridSize[i];
  }
  prop->numBarriers = 16;
  prop->totalGlobalMem = p.totalGlobalMem;
  prop->sharedMemPerMultiprocessor = p.sharedMemPerMultiprocessor;
  prop->sharedMemPerBlock = p.sharedMemPerBlockOptin;
  prop->memBankCount = 32;
  prop->memBankSize = 4;
  prop->cacheLineSize = 128;
  int clk_khz = 0, mem_khz = 0;
  cudaDeviceGetAttribute(&clk_khz, cudaDevAttrClockRate, device);
  cudaDeviceGetAttribute(&mem_khz, cudaDevAttrMemoryClockRate, device);
  prop->clockRateMHz = clk_khz / 1000;
  // DDR: two transfers per clock over the bus width.
  prop->peakMemoryBandwidthMBs = (size_t)((double)mem_khz * 1e3 * 2.0 * (p.memoryBusWidth / 8) / 1e6);
  prop->unifiedAddressing = p.unifiedAddressing;
  prop->managedMemory = p.managedMemory;
  prop->warpShuffleIsEmulated = 0;
  prop->eventTimingIsDeviceSide = 1;
  prop->constantMemoryIsGlobal = 0;
  return grxSuccess;
}

grxError_t grxDeviceSynchronize(void) { return rec(cudaDeviceSynchronize()); }

grxError_t grxMemGetInfo(size_t* f, size_t* t) {
  if (!f || !t) return rec_g(grxErrorInvalidValue);
  return rec(cudaMemGetInfo(f, t));
}

grxError_t grxDeviceCanAccessPeer(int* can, int device, int peer) {
  if (!can) return rec_g(grxErrorInvalidValue);
  return rec(cudaDeviceCanAccessPeer(can, device, peer));
}

grxError_t grxDeviceEnablePeerAccess(int peer, unsigned int flags) {
  const cudaError_t e = cudaDeviceEnablePeerAccess(peer, flags);
  if (e == cudaErrorPeerAccessAlreadyEnabled) {
    cudaGetLastError();
    return grxSuccess;
  }
  return rec(e);
}

grxError_t grxIpcGetMemHandle(grxIpcMemHandle_t* handle, void* dev_ptr) {
  static_assert(sizeof(grxIpcMemHandle_t) == sizeof(cudaIpcMemHandle_t), "IPC handle size");
  if (!handle || !dev_ptr) return rec(cudaErrorInvalidValue);
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, dev_ptr);
  if (e == cudaSuccess) memcpy(handle, &h, sizeof(h));
  return rec(e);
}

grxError_t grxIpcOpenMemHandle(void** dev_ptr, grxIpcMemHandle_t handle) {
  if (!dev_ptr) return rec(cudaErrorInvalidValue);
  cudaIpcMemHandle_t h;
  memcpy(&h, &handle, sizeof(h));
  return rec(cudaIpcOpenMemHandle(dev_ptr, h, cudaIpcMemLazyEnablePeerAccess));
}

grxError_t grxIpcCloseMemHandle(void* dev_ptr) { return rec(cudaIpcCloseMemHandle(dev_ptr)); }

grxError_t grxGetLastError(void) {
  const grxError_t e = g_last_error;
  g_last_error = grxSuccess;
  return e;
}
grxError_t grxPeekAtLastError(void) { return g_last_error; }

grxError_t grxMalloc(void** ptr, size_t size) {
  if (!ptr) return rec_g(grxErrorInvalidValue);
  return rec(cudaMalloc(ptr, size));
}
grxError_t grxFree(void* ptr) { return rec(cudaFree(ptr)); }
grxError_t grxMallocHost(void** ptr, size_t size) {
  if (!ptr) return rec_g(grxErrorInvalidValue);
  return rec(cudaMallocHost(ptr, size));
}
grxError_t grxFreeHost(void* ptr) { return rec(cudaFreeHost(ptr)); }

static cudaMemcpyKind kind_of(grxMemcpyKind k) {
  switch (k) {
    case grxMemcpyHostToHost: return cudaMemcpyHostToHost;
    case grxMemcpyHostToDevice: return cudaMemcpyHostToDevice;
    case grxMemcpyDeviceToHost: return cudaMemcpyDeviceToHost;
    case grxMemcpyDeviceToDevice: return cudaMemcpyDeviceToDevice;
    default: return cudaMemcpyDefault;
  }
}

grxError_t grxMemcpy(void* dst, const void* src, size_t count, grxMemcpyKind kind) {
  if ((unsigned)kind > 4u) return rec_g(grxErrorInvalidMemcpyDirection);
  return rec(cudaMemcpy(dst, src, count, kind_of(kind)));
}
grxError_t grxMemcpyAsync(void* dst, const void* src, size_t count, grxMemcpyKind kind, grxStream_t s) {
  if ((unsigned)kind > 4u) return rec_g(grxErrorInvalidMemcpyDirection);
  return rec(cudaMemcpyAsync(dst, src, count, kind_of(kind), cs(s)));
}
grxError_t grxMemset(void* dst, int value, size_t count) { return rec(cudaMemset(dst, value, count)); }
grxError_t grxMemsetAsync(void* dst, int value, size_t count, grxStream_t s) {
  return rec(cudaMemsetAsync(dst, value, count, cs(s)));
}

grxError_t grxStreamCreate(grxStream_t* s) { return grxStreamCreateWithFlags(s, grxStreamDefault); }
grxError_t grxStreamCreateWithFlags(grxStream_t* s, unsigned int flags) {
  if (!s) return rec_g(grxErrorInvalidValue);
  cudaStream_t st = nullptr;
  const cudaError_t e =
      cudaStreamCreateWithFlags(&st, (flags & grxStreamNonBlocking) ? cudaStreamNonBlocking : cudaStreamDefault);
  *s = reinterpret_cast<grxStream_t>(st);
  return rec(e);
}
grxError_t grxStreamDestroy(grxStream_t s) { return rec(cudaStreamDestroy(cs(s))); }
grxError_t grxStreamSynchronize(grxStream_t s) { return rec(cudaStreamSynchronize(cs(s))); }
grxError_t grxStreamQuery(grxStream_t s) {
  const cudaError_t e = cudaStreamQuery(cs(s));
  if (e == cudaErrorNotReady) {
    cudaGetLastError();
    return grxErrorNotReady;
  }
  return rec(e);
}
grxError_t grxStreamWaitEvent(grxStream_t s, grxEvent_t ev, unsigned int flags) {
  return rec(cudaStreamWaitEvent(cs(s), ce(ev), flags));
}

grxError_t grxEventCreate(grxEvent_t* ev) { return grxEventCreateWithFlags(ev, grxEventDefault); }
grxError_t grxEventCreateWithFlags(grxEvent_t* ev, unsigned int flags) {
  if (!ev) return rec_g(grxErrorInvalidValue);
  unsigned f = cudaEventDefault;
  if (flags & grxEventBlockingSync) f |= cudaEventBlockingSync;
  if (flags & grxEventDisableTiming) f |= cudaEventDisableTiming;
  cudaEvent_t e = nullptr;
  const cudaError_t r = cudaEventCreateWithFlags(&e, f);
  *ev = reinterpret_cast<grxEvent_t>(e);
  return rec(r);
}
grxError_t grxEventDestroy(grxEvent_t ev) { return rec(cudaEventDestroy(ce(ev))); }
grxError_t grxEventRecord(grxEvent_t ev, grxStream_t s) { return rec(cudaEventRecord(ce(ev), cs(s))); }
grxError_t grxEventSynchronize(grxEvent_t ev) { return rec(cudaEventSynchronize(ce(ev))); }
grxError_t grxEventQuery(grxEvent_t ev) {
  const cudaError_t e = cudaEventQuery(ce(ev));
  if (e == cudaErrorNotReady) {
    cudaGetLastError();
    return grxErrorNotReady;
  }
  return rec(e);
}
grxError_t grxEventElapsedTime(float* ms, grxEvent_t a, grxEvent_t b) {
  if (!ms) return rec_g(grxErrorInvalidValue);
  return rec(cudaEventElapsedTime(ms, ce(a), ce(b)));
}

// Tensor maps (reference grx_tensormap.h:78-108). B200 has no descriptor slots:
// a TMA descriptor is a per-launch kernel parameter, so there is nothing to
// program and the slot count is 0.
grxError_t grxTensorMapGetSlotCount(int* count, int device) {
  if (!count) return rec_g(grxErrorInvalidValue);
  int n = 0;
  const cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess) return rec(e);
  if (device < 0 || device >= n) return rec_g(grxErrorInvalidDevice);
  *count = 0;
  return grxSuccess;
}
grxError_t grxMallocPhysical(void** ptr, size_t size) { return grxMalloc(ptr, size); }
grxError_t grxTensorMapProgramAsync(const grxTensorMapDesc_t* desc, grxStream_t) {
  if (!desc) return rec_g(grxErrorInvalidValue);
  return rec_g(grxErrorNotSupported);
}
grxError_t grxTensorMapProgram(const grxTensorMapDesc_t* desc) { return grxTensorMapProgramAsync(desc, nullptr); }

}  // extern "C"
