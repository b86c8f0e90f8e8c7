#include "profile.h"

#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

#include <mutex>

#include "host_common.h"

namespace grx {

namespace {

std::mutex g_mu;
unsigned long long g_seq = 0;
bool g_device_announced = false;

unsigned long long host_ns() {
  timespec ts;
  clock_gettime(CLOCK_MONOTONIC, &ts);
  return (unsigned long long)ts.tv_sec * 1000000000ull + (unsigned long long)ts.tv_nsec;
}

void announce_device_locked() {
  if (g_device_announced) return;
  g_device_announced = true;
  int dev = 0;
  cudaGetDevice(&dev);
  cudaDeviceProp p;
  if (cudaGetDeviceProperties(&p, dev) != cudaSuccess) {
    cudaGetLastError();
    return;
  }
  int clk_khz = 0;
  cudaDeviceGetAttribute(&clk_khz, cudaDevAttrClockRate, dev);
  fprintf(stderr,
          "GRXPROF|device|name=%s|backend=silicon|cores=%d|warps_per_core=%d|warp_size=%d|shared_per_sm=%zu"
          "|clock_mhz=%d|event_timing_is_device_side=1\n",
          p.name, p.multiProcessorCount, p.maxThreadsPerMultiProcessor / p.warpSize, p.warpSize,
          (size_t)p.sharedMemPerMultiprocessor, clk_khz / 1000);
}

}  // namespace

bool profile_enabled() {
  static const bool on = [] {
    const char* v = getenv("GRX_PROFILE");
    return v && v[0] && strcmp(v, "0") != 0;
  }();
  return on;
}

ProfLaunch::ProfLaunch(const char* kernel, dim3 grid, dim3 block, size_t shared, cudaStream_t stream)
    : kernel_(kernel), grid_(grid), block_(block), shared_(shared), stream_(stream) {
  if (!profile_enabled()) return;
  // The sync makes the measurement attributable to this launch alone, as in
  // the reference (profile_begin syncs every stream of the device).
  if (cudaDeviceSynchronize() != cudaSuccess) {
    cudaGetLastError();
    return;
  }
  if (cudaEventCreate(&e0_) != cudaSuccess || cudaEventCreate(&e1_) != cudaSuccess) {
    cudaGetLastError();
    return;
  }
  host_start_ns_ = host_ns();
  cudaEventRecord(e0_, stream_);
  on_ = true;
}

ProfLaunch::~ProfLaunch() {
  if (!on_) return;
  cudaEventRecord(e1_, stream_);
  const cudaError_t e = cudaDeviceSynchronize();
  const unsigned long long host_end = host_ns();
  float ms = -1.f;
  if (e == cudaSuccess) cudaEventElapsedTime(&ms, e0_, e1_);
  cudaGetLastError();
  cudaEventDestroy(e0_);
  cudaEventDestroy(e1_);
  std::lock_guard<std::mutex> lock(g_mu);
  announce_device_locked();
  fprintf(stderr,
          "GRXPROF|1|op=launch|seq=%llu|kernel=%s|module=%s|stream=%llu|grid=%u.%u.%u|block=%u.%u.%u|shared=%zu"
          "|host_start_ns=%llu|host_end_ns=%llu|c.device_ns=%lld\n",
          g_seq++, kernel_, library_path(), (unsigned long long)(uintptr_t)stream_, grid_.x, grid_.y, grid_.z,
          block_.x, block_.y, block_.z, shared_, host_start_ns_, host_end,
          ms >= 0.f ? (long long)((double)ms * 1e6) : -1LL);
}

}  // namespace grx
