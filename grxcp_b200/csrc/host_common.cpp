#include "host_common.h"

#include <dlfcn.h>
#include <limits.h>
#include <stdlib.h>
#include <string.h>

#include <mutex>
#include <string>

#include "kernels.h"

namespace grx {

bool fault_injected(const char* site) {
  const char* e = getenv("GRX_FAULT_INJECT");
  if (!e || !*e) return false;
  const size_t n = strlen(site);
  for (const char* p = e; *p;) {
    const char* end = strchr(p, ',');
    const size_t len = end ? (size_t)(end - p) : strlen(p);
    if (len == n && strncmp(p, site, n) == 0) return true;
    if (!end) break;
    p = end + 1;
  }
  return false;
}

int ensure_device(DeviceState& d) {
  if (d.device >= 0) return 0;
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    return 1;
  }
  cudaDeviceProp p;
  if (cudaGetDeviceProperties(&p, dev) != cudaSuccess) {
    cudaGetLastError();
    return 1;
  }
  int* w = nullptr;
  if (fault_injected("alloc")) return 2;
  if (cudaMalloc(&w, sizeof(int)) != cudaSuccess) {
    cudaGetLastError();
    return 2;
  }
  if (cudaMemset(w, 0, sizeof(int)) != cudaSuccess) {
    cudaFree(w);
    cudaGetLastError();
    return 2;
  }
  d.device = dev;
  d.cc_major = p.major;
  d.num_sms = p.multiProcessorCount;
  d.err_word = w;
  return 0;
}

void release_device(DeviceState& d) {
  if (d.err_word) cudaFree(d.err_word);
  d = DeviceState{};
}

int take_error(DeviceState& d, cudaStream_t stream) {
  if (!d.err_word) return 0;
  if (cudaStreamSynchronize(stream) != cudaSuccess) {
    cudaGetLastError();
    return -1;
  }
  int code = 0;
  if (cudaMemcpy(&code, d.err_word, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) {
    cudaGetLastError();
    return -1;
  }
  if (code != 0) cudaMemset(d.err_word, 0, sizeof(int));
  return code;
}

unsigned long long wait_timeout_ns() {
  static unsigned long long ns = [] {
    const char* e = getenv("GRX_WAIT_TIMEOUT_MS");
    long long ms = e ? atoll(e) : 2000;
    if (ms <= 0) ms = 2000;
    return (unsigned long long)ms * 1000000ull;
  }();
  return ns;
}

static void marker() {}

const char* library_path() {
  static std::string path;
  static std::once_flag once;
  std::call_once(once, [] {
    Dl_info info;
    if (dladdr(reinterpret_cast<void*>(&marker), &info) && info.dli_fname) {
      char buf[PATH_MAX];
      path = realpath(info.dli_fname, buf) ? std::string(buf) : std::string(info.dli_fname);
    }
  });
  return path.c_str();
}

bool path_names_library(const char* cfg) {
  char buf[PATH_MAX];
  if (!realpath(cfg, buf)) return false;
  const std::string p(buf), lib(library_path());
  if (p == lib) return true;
  const size_t slash = lib.rfind('/');
  return slash != std::string::npos && p == lib.substr(0, slash);
}

}  // namespace grx

// Internal test entry point (not part of the grx* API): runs the bounded-wait
// probe kernel and returns the error code it left (expected: 5, a timeout), or
// -1 on a launch/runtime failure.
extern "C" int grxcpTestBoundedWait(unsigned long long timeout_ns) {
  int* w = nullptr;
  if (cudaMalloc(&w, sizeof(int)) != cudaSuccess) return -1;
  cudaMemset(w, 0, sizeof(int));
  int code = -1;
  if (grx::launch_bounded_wait_probe(w, timeout_ns, nullptr) == cudaSuccess && cudaDeviceSynchronize() == cudaSuccess)
    cudaMemcpy(&code, w, sizeof(int), cudaMemcpyDeviceToHost);
  cudaFree(w);
  return code;
}
