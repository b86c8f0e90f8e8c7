/* Host-side stand-in for the GRX-G100 device environment, so the reference's
 * sgemm kernel source (src/libs/grxblas/kernels/sgemm.cpp) compiles unchanged
 * as ordinary host C++ for use as a test oracle. Provides what that file uses:
 * __global__, __UNIFORM__, blockIdx / blockDim / threadIdx, and a no-op
 * grx::cycle_probe. The driver (oracle/ref_sgemm_driver.cpp) walks the grid
 * serially, setting these before each call. TEST INFRASTRUCTURE ONLY. */
#pragma once
#include <stdint.h>

#define __global__
#define __UNIFORM__

struct grx_ref_dim3 { uint32_t x, y, z; };
extern thread_local grx_ref_dim3 blockIdx, blockDim, threadIdx, gridDim;

typedef struct { uint64_t start, end; uint32_t core, warp; } grxCycleSlot;

namespace grx {
class cycle_probe {
 public:
  explicit cycle_probe(grxCycleSlot*) {}
  void finish() {}
};
}  // namespace grx
