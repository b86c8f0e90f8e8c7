// Host-side plumbing shared by the grxBLAS and grxDNN handles.
#pragma once

#include <cuda_runtime.h>

namespace grx {

// Per-handle device binding, made on first use: the device current at that
// moment, its SM count and compute capability, and a device word that kernels
// launched through the handle write an error code into when a bounded wait
// gives up.
struct DeviceState {
  int device = -1;
  int cc_major = 0;
  int num_sms = 0;
  int* err_word = nullptr;
};

// 0 ok, 1 no usable CUDA device, 2 allocation failed.
int ensure_device(DeviceState& d);
void release_device(DeviceState& d);

// Synchronises `stream`, returns and clears the error word (>= 0), or -1 if
// the stream itself reported an error.
int take_error(DeviceState& d, cudaStream_t stream);

// Bounded-wait limit for every kernel (GRX_WAIT_TIMEOUT_MS, default 2000 ms).
unsigned long long wait_timeout_ns();

// Absolute path of this shared library (the file the kernels run from).
const char* library_path();

// True when `path` names this library file or the directory holding it.
bool path_names_library(const char* path);

// Host-side fault injection. GRX_FAULT_INJECT holds a comma-separated list of
// sites whose next call this library treats as failed, read on every check:
//   alloc      every device allocation the library makes (error word,
//              workspace): the API returns ALLOC_FAILED
//   module     kernel-path resolution (GRXBLAS_KERNEL_PATH rule): the API
//              returns NOT_INITIALIZED, as when the kernels are not found
//   nccl_init  communicator creation in grxblasShardCommInit: EXECUTION_FAILED
//   nccl_load  loading libnccl: NOT_SUPPORTED
// Nothing is injected on the device: no kernel is made to fault or hang.
bool fault_injected(const char* site);

}  // namespace grx
