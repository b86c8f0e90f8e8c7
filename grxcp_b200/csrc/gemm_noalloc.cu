// grxblasGemmExNoAlloc: the tensor-core GemmEx for callers that may not
// allocate device memory.
//
// Some callers can't call cudaMalloc: a process whose device memory is owned
// by another allocator (a framework plug-in inside a caching allocator, a
// serving process with a fixed memory budget fixed at start-up), or a caller
// that must not pay the implicit device-wide synchronisation cudaMalloc and
// cudaFree can bring. grxblasGemmEx may allocate twice: the handle's error word
// on first use, and its workspace when an operand has to be packed (address,
// leading dimension not 16-byte aligned). This entry point allocates nothing.
// It takes no handle; its packing scratch is the file-scope array below, and
// the bounded-wait error flag is an optional caller-owned device int.
//
// The scratch array is a fixed-size __device__ object: every GPU that loads
// this library holds kNoAllocScratchBytes of it until the process exits.
// Problems whose packed operands need more are refused (INVALID_VALUE, with a
// line on stderr naming the limit). Every call shares the array and it keeps
// the last call's contents; the packer rewrites every byte the GEMM then reads
// (the k padding included), so nothing relies on it starting at zero. Calls
// that overlap on the GPU (different streams, no ordering between them) race
// on the array; callers must order them.
//
// Host code cannot use the array's name as a device address (in host code it
// names a host-side stand-in). The first call on each device, with that device
// current, resolves the address once with cudaGetSymbolAddress, checks the
// result and caches it; make that first call before any stream capture.
#include <cuda_runtime.h>
#include <stdio.h>

#include <mutex>

#include "gemm_tc.cuh"
#include "grx/grxblas.h"
#include "host_common.h"
#include "kernels.h"

namespace {

constexpr size_t kNoAllocScratchBytes = 16u << 20;  // 16 MiB for both packed operands

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

struct DeviceSlot {
  bool ready = false;
  unsigned char* scratch = nullptr;  // device address of g_noalloc_scratch on this device
  int num_sms = 0;
  int cc_major = 0;
};

constexpr int kMaxDevices = 64;
std::mutex g_mu;
DeviceSlot g_slots[kMaxDevices];

// Once per device, with that device current: resolve the scratch address.
grxblasStatus_t setup_current_device(DeviceSlot& out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    cudaGetLastError();
    return GRXBLAS_STATUS_NOT_INITIALIZED;
  }
  std::lock_guard<std::mutex> lock(g_mu);
  DeviceSlot& s = g_slots[dev];
  if (!s.ready) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) {
      cudaGetLastError();
      return GRXBLAS_STATUS_NOT_INITIALIZED;
    }
    int sms = 0, major = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess) {
      cudaGetLastError();
      return GRXBLAS_STATUS_NOT_INITIALIZED;
    }
    s.scratch = static_cast<unsigned char*>(p);
    s.num_sms = sms;
    s.cc_major = major;
    s.ready = true;
  }
  out = s;
  return GRXBLAS_STATUS_SUCCESS;
}

grxblasStatus_t status_of(cudaError_t e) {
  switch (e) {
    case cudaSuccess: return GRXBLAS_STATUS_SUCCESS;
    case cudaErrorInvalidValue: return GRXBLAS_STATUS_INVALID_VALUE;
    case cudaErrorNotSupported: return GRXBLAS_STATUS_NOT_SUPPORTED;
    default: return GRXBLAS_STATUS_EXECUTION_FAILED;
  }
}

long long up(long long v, long long a) { return (v + a - 1) / a * a; }

}  // namespace

extern "C" grxblasStatus_t grxblasGemmExNoAlloc(grxStream_t stream, grxblasOperation_t transa,
                                                grxblasOperation_t transb, int m, int n, int k, const float* alpha,
                                                const void* A, grxDataType_t Atype, int lda, const void* B,
                                                grxDataType_t Btype, int ldb, const float* beta, void* C,
                                                grxDataType_t Ctype, int ldc, int* errorFlag) {
  // Argument rules of grxblasGemmEx (reference grxblas.cpp:506-524).
  if (!alpha || !beta) return GRXBLAS_STATUS_INVALID_VALUE;
  if (m < 0 || n < 0 || k < 0) return GRXBLAS_STATUS_INVALID_VALUE;
  if (m == 0 || n == 0) return GRXBLAS_STATUS_SUCCESS;
  if (k > 0 && (!A || !B)) return GRXBLAS_STATUS_INVALID_VALUE;
  if (!C) return GRXBLAS_STATUS_INVALID_VALUE;
  const bool ta = transa == GRXBLAS_OP_T, tb = transb == GRXBLAS_OP_T;
  if (lda < (ta ? k : m) || ldb < (tb ? n : k) || ldc < m) return GRXBLAS_STATUS_INVALID_VALUE;

  int kind, out, fmt, es;
  if (Atype != Btype) return GRXBLAS_STATUS_NOT_SUPPORTED;
  if (Atype == GRX_R_16F && (Ctype == GRX_R_32F || Ctype == GRX_R_16F)) {
    kind = grx::kKindF16; fmt = 0; es = 2; out = Ctype == GRX_R_32F ? grx::kOutF32 : grx::kOutF16;
  } else if (Atype == GRX_R_16BF && (Ctype == GRX_R_32F || Ctype == GRX_R_16BF)) {
    kind = grx::kKindF16; fmt = 1; es = 2; out = Ctype == GRX_R_32F ? grx::kOutF32 : grx::kOutBF16;
  } else if (Atype == GRX_R_8I && (Ctype == GRX_R_32I || Ctype == GRX_R_16BF || Ctype == GRX_R_32F)) {
    kind = grx::kKindI8; fmt = 1; es = 1;
    out = Ctype == GRX_R_32I ? grx::kOutS32 : (Ctype == GRX_R_16BF ? grx::kOutBF16 : grx::kOutF32);
    // The exact int32 output takes integer alpha/beta only (reference
    // grxblas.cpp:580-584); the float outputs take any.
    const float a = *alpha, b = *beta;
    if (out == grx::kOutS32 && (a != (float)(int)a || b != (float)(int)b)) return GRXBLAS_STATUS_INVALID_VALUE;
  } else if (Atype == GRX_R_8F_E4M3 && (Ctype == GRX_R_32F || Ctype == GRX_R_16BF)) {
    kind = grx::kKindF8; fmt = 0; es = 1; out = Ctype == GRX_R_32F ? grx::kOutF32 : grx::kOutBF16;
  } else {
    return GRXBLAS_STATUS_NOT_SUPPORTED;
  }

  DeviceSlot dev;
  const grxblasStatus_t st = setup_current_device(dev);
  if (st != GRXBLAS_STATUS_SUCCESS) return st;
  if (dev.cc_major != 10) return GRXBLAS_STATUS_ARCH_MISMATCH;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);

  if (k == 0)
    return status_of(grx::launch_gemm_k0(out, C, ldc, 0, m, n, 1, *beta, (int)*beta, nullptr, 0, 0, 0, 0, s));

  // Operands TMA cannot read as stored are packed K-major into the static scratch.
  const bool pack_a = !grx::tma_operand_ok(A, lda, 0, es, 1);
  const bool pack_b = !grx::tma_operand_ok(B, ldb, 0, es, 1);
  const long long ldp = up(k, 16 / es);
  const size_t bytes_a = pack_a ? (size_t)up((long long)m * ldp * es, 256) : 0;
  const size_t bytes_b = pack_b ? (size_t)up((long long)n * ldp * es, 256) : 0;
  if (bytes_a + bytes_b > kNoAllocScratchBytes) {
    fprintf(stderr,
            "grxblas: grxblasGemmExNoAlloc needs %zu bytes of packing scratch for this problem; its fixed "
            "scratch holds %zu. Align the operands to 16 bytes (address and leading dimension) or call "
            "grxblasGemmEx.\n",
            bytes_a + bytes_b, kNoAllocScratchBytes);
    return GRXBLAS_STATUS_INVALID_VALUE;
  }

  grx::TcGemmLaunch L{};
  L.kind = kind;
  L.out = out;
  L.a_fmt = fmt;
  L.a = A; L.lda = lda; L.stride_a = 0; L.a_mn_major = ta ? 0 : 1;
  L.b = B; L.ldb = ldb; L.stride_b = 0; L.b_mn_major = tb ? 1 : 0;
  if (pack_a) {
    cudaError_t e = grx::launch_pack_kmajor(A, es, ta ? 0 : 1, lda, 0, 1, m, k, dev.scratch, ldp, s);
    if (e != cudaSuccess) return status_of(e);
    L.a = dev.scratch; L.lda = ldp; L.a_mn_major = 0;
  }
  if (pack_b) {
    unsigned char* wb = dev.scratch + bytes_a;
    cudaError_t e = grx::launch_pack_kmajor(B, es, tb ? 1 : 0, ldb, 0, 1, n, k, wb, ldp, s);
    if (e != cudaSuccess) return status_of(e);
    L.b = wb; L.ldb = ldp; L.b_mn_major = 0;
  }
  grx::TcGemmParams& p = L.p;
  p.m = m; p.n = n; p.k = k; p.batch = 1;
  p.alpha = *alpha; p.beta = *beta;
  p.ialpha = (int)*alpha; p.ibeta = (int)*beta;
  p.beta_nonzero = *beta != 0.0f;
  p.c = C; p.ldc = ldc; p.stride_c = 0;
  p.err_word = errorFlag;
  p.timeout_ns = grx::wait_timeout_ns();
  p.group_m = 16;
  return status_of(grx::launch_tc_gemm(L, dev.num_sms, s));
}
