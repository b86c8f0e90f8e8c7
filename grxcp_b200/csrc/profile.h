// GRX_PROFILE launch tracing, in the reference's GRXPROF line format
// (src/runtime/profile.cpp:147-290): with GRX_PROFILE set (and not "0"),
// every kernel launch of this library is bracketed by device synchronisations
// and reported on stderr as
//   GRXPROF|1|op=launch|seq=..|kernel=..|module=..|stream=..|grid=x.y.z
//     |block=x.y.z|shared=..|host_start_ns=..|host_end_ns=..|c.device_ns=..
// preceded once per process by a GRXPROF|device|... line. The counter field is
// the launch's device time from CUDA events (the reference reports hardware
// performance-monitor deltas in the same |c.name=value form). Off by default;
// when off, a launch pays one cached boolean test.
#pragma once

#include <cuda_runtime.h>

namespace grx {

bool profile_enabled();

class ProfLaunch {
 public:
  ProfLaunch(const char* kernel, dim3 grid, dim3 block, size_t shared, cudaStream_t stream);
  ~ProfLaunch();
  ProfLaunch(const ProfLaunch&) = delete;
  ProfLaunch& operator=(const ProfLaunch&) = delete;

 private:
  bool on_ = false;
  const char* kernel_;
  dim3 grid_, block_;
  size_t shared_;
  cudaStream_t stream_;
  cudaEvent_t e0_ = nullptr, e1_ = nullptr;
  unsigned long long host_start_ns_ = 0;
};

}  // namespace grx
