// Column-parallel grxBLAS over NCCL, for C/C++ callers (no counterpart in the
// reference, which runs on one device).
//
// One process per GPU. Rank 0 makes an NCCL unique id (grxblasShardGetUniqueId)
// and hands it to the other ranks out of band (a file, a socket, MPI); every
// rank then creates its communicator on its current device
// (grxblasShardCommInit). grxblasGemmExColumnParallel runs this rank's share of
// the columns of C = alpha op(A) op(B) + beta C as one local GemmEx on the
// handle's stream, and with replicate != 0 every rank broadcasts its column
// block in one NCCL group, so C ends up complete on every rank.
//
// Failure detection stays on the host. The communicator is non-blocking
// (ncclConfig_t.blocking = 0): creation and every enqueue are polled with
// ncclCommGetAsyncError against a deadline, and grxblasShardSynchronize waits
// for the stream the same way. When the deadline passes (a rank that never
// joins, or one that left between steps) the communicator is aborted with
// ncclCommAbort and the call returns EXECUTION_FAILED; the communicator is then
// unusable and must be destroyed. The deadline is GRX_SHARD_TIMEOUT_MS
// (default 60000). libnccl is loaded at first use with dlopen (an NCCL already
// loaded into the process, e.g. by torch, is reused), so the library itself
// does not depend on it.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

#include <mutex>

#include "grx/grxblas.h"
#include "host_common.h"

namespace grx {
// blas_host.cpp: GemmEx over columns [col0, col0 + n) of a wider problem (the
// handle's per-column bias and scales are offset by col0).
grxblasStatus_t gemm_ex_columns(grxblasHandle_t handle, grxblasOperation_t transa, grxblasOperation_t transb, int m,
                                int n, int k, const float* alpha, const void* A, grxDataType_t Atype, int lda,
                                const void* B, grxDataType_t Btype, int ldb, const float* beta, void* C,
                                grxDataType_t Ctype, int ldc, long long col0);
}  // namespace grx

struct grxblasShardContext {
  ncclComm_t comm = nullptr;
  int rank = 0, world = 1, device = -1;
  bool broken = false;  // aborted after a deadline: only destroy is allowed
};

namespace {

struct NcclApi {
  bool ok = false;
  ncclResult_t (*GetUniqueId)(ncclUniqueId*);
  ncclResult_t (*CommInitRankConfig)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*);
  ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*);
  ncclResult_t (*CommAbort)(ncclComm_t);
  ncclResult_t (*CommDestroy)(ncclComm_t);
  ncclResult_t (*CommFinalize)(ncclComm_t);
  ncclResult_t (*Broadcast)(const void*, void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t);
  ncclResult_t (*GroupStart)();
  ncclResult_t (*GroupEnd)();
};

NcclApi load_nccl() {
  NcclApi a{};
  void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
  if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
  if (!h) return a;
  bool all = true;
  auto sym = [&](const char* name) {
    void* f = dlsym(h, name);
    all = all && f != nullptr;
    return f;
  };
  a.GetUniqueId = reinterpret_cast<decltype(a.GetUniqueId)>(sym("ncclGetUniqueId"));
  a.CommInitRankConfig = reinterpret_cast<decltype(a.CommInitRankConfig)>(sym("ncclCommInitRankConfig"));
  a.CommGetAsyncError = reinterpret_cast<decltype(a.CommGetAsyncError)>(sym("ncclCommGetAsyncError"));
  a.CommAbort = reinterpret_cast<decltype(a.CommAbort)>(sym("ncclCommAbort"));
  a.CommDestroy = reinterpret_cast<decltype(a.CommDestroy)>(sym("ncclCommDestroy"));
  a.CommFinalize = reinterpret_cast<decltype(a.CommFinalize)>(sym("ncclCommFinalize"));
  a.Broadcast = reinterpret_cast<decltype(a.Broadcast)>(sym("ncclBroadcast"));
  a.GroupStart = reinterpret_cast<decltype(a.GroupStart)>(sym("ncclGroupStart"));
  a.GroupEnd = reinterpret_cast<decltype(a.GroupEnd)>(sym("ncclGroupEnd"));
  a.ok = all;
  return a;
}

const NcclApi* nccl() {
  if (grx::fault_injected("nccl_load")) return nullptr;
  static NcclApi api = load_nccl();
  return api.ok ? &api : nullptr;
}

long long deadline_ms() {
  const char* e = getenv("GRX_SHARD_TIMEOUT_MS");
  const long long v = e ? atoll(e) : 60000;
  return v > 0 ? v : 60000;
}

double now_ms() {
  timespec ts;
  clock_gettime(CLOCK_MONOTONIC, &ts);
  return ts.tv_sec * 1e3 + ts.tv_nsec * 1e-6;
}

void nap() {
  timespec ts{0, 200000};  // 0.2 ms
  nanosleep(&ts, nullptr);
}

// Polls the communicator until its pending operation leaves ncclInProgress.
// Past the deadline: abort, mark broken, EXECUTION_FAILED.
grxblasStatus_t settle(grxblasShardContext& c, ncclResult_t r, double t0) {
  const NcclApi* n = nccl();
  while (r == ncclInProgress) {
    if (now_ms() - t0 > (double)deadline_ms()) {
      n->CommAbort(c.comm);
      c.comm = nullptr;
      c.broken = true;
      return GRXBLAS_STATUS_EXECUTION_FAILED;
    }
    nap();
    if (n->CommGetAsyncError(c.comm, &r) != ncclSuccess) r = ncclInternalError;
  }
  if (r != ncclSuccess) {
    n->CommAbort(c.comm);
    c.comm = nullptr;
    c.broken = true;
    return GRXBLAS_STATUS_EXECUTION_FAILED;
  }
  return GRXBLAS_STATUS_SUCCESS;
}

size_t elem_bytes(grxDataType_t t) {
  switch (t) {
    case GRX_R_32F:
    case GRX_R_32I: return 4;
    case GRX_R_16F:
    case GRX_R_16BF: return 2;
    case GRX_R_8I:
    case GRX_R_8F_E4M3: return 1;
    default: return 0;
  }
}

}  // namespace

extern "C" {

grxblasStatus_t grxblasShardRange(int n, int rank, int world, int* start, int* count) {
  if (!start || !count || n < 0 || world <= 0 || rank < 0 || rank >= world) return GRXBLAS_STATUS_INVALID_VALUE;
  const int base = n / world, extra = n % world;
  *start = rank * base + (rank < extra ? rank : extra);
  *count = base + (rank < extra ? 1 : 0);
  return GRXBLAS_STATUS_SUCCESS;
}

grxblasStatus_t grxblasShardGetUniqueId(grxblasShardUniqueId_t* id) {
  static_assert(sizeof(grxblasShardUniqueId_t) == sizeof(ncclUniqueId), "unique id size");
  if (!id) return GRXBLAS_STATUS_INVALID_VALUE;
  const NcclApi* n = nccl();
  if (!n) return GRXBLAS_STATUS_NOT_SUPPORTED;
  ncclUniqueId u;
  if (n->GetUniqueId(&u) != ncclSuccess) return GRXBLAS_STATUS_EXECUTION_FAILED;
  memcpy(id->internal, u.internal, sizeof(u.internal));
  return GRXBLAS_STATUS_SUCCESS;
}

grxblasStatus_t grxblasShardCommInit(grxblasShardComm_t* comm, const grxblasShardUniqueId_t* id, int rank,
                                     int world) {
  if (!comm || !id || world <= 0 || rank < 0 || rank >= world) return GRXBLAS_STATUS_INVALID_VALUE;
  *comm = nullptr;
  const NcclApi* n = nccl();
  if (!n) return GRXBLAS_STATUS_NOT_SUPPORTED;
  if (grx::fault_injected("nccl_init")) return GRXBLAS_STATUS_EXECUTION_FAILED;
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    return GRXBLAS_STATUS_NOT_INITIALIZED;
  }
  auto* c = new grxblasShardContext;
  c->rank = rank;
  c->world = world;
  c->device = dev;
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;
  ncclUniqueId u;
  memcpy(u.internal, id->internal, sizeof(u.internal));
  const double t0 = now_ms();
  ncclResult_t r = n->CommInitRankConfig(&c->comm, world, u, rank, &cfg);
  if (r != ncclSuccess && r != ncclInProgress) {
    if (c->comm) n->CommAbort(c->comm);
    delete c;
    return GRXBLAS_STATUS_EXECUTION_FAILED;
  }
  if (r == ncclInProgress || r == ncclSuccess) {
    ncclResult_t a = ncclInProgress;
    if (n->CommGetAsyncError(c->comm, &a) != ncclSuccess) a = ncclInternalError;
    const grxblasStatus_t st = settle(*c, a, t0);
    if (st != GRXBLAS_STATUS_SUCCESS) {
      delete c;
      return st;
    }
  }
  *comm = c;
  return GRXBLAS_STATUS_SUCCESS;
}

grxblasStatus_t grxblasShardCommDestroy(grxblasShardComm_t comm) {
  if (!comm) return GRXBLAS_STATUS_SUCCESS;
  const NcclApi* n = nccl();
  if (comm->comm && n) {
    // finalize flushes pending work (non-blocking: poll it), then destroy
    const double t0 = now_ms();
    ncclResult_t r = n->CommFinalize(comm->comm);
    const grxblasStatus_t st = settle(*comm, r == ncclSuccess ? ncclInProgress : r, t0);
    if (st == GRXBLAS_STATUS_SUCCESS && comm->comm) n->CommDestroy(comm->comm);
  }
  delete comm;
  return GRXBLAS_STATUS_SUCCESS;
}

grxblasStatus_t grxblasGemmExColumnParallel(grxblasHandle_t handle, grxblasShardComm_t comm,
                                            grxblasOperation_t transa, grxblasOperation_t transb, int m, int n, int k,
                                            const float* alpha, const void* A, grxDataType_t Atype, int lda,
                                            const void* B, grxDataType_t Btype, int ldb, const float* beta, void* C,
                                            grxDataType_t Ctype, int ldc, int replicate) {
  if (!handle) return GRXBLAS_STATUS_NOT_INITIALIZED;
  if (!comm) return GRXBLAS_STATUS_INVALID_VALUE;
  if (comm->broken) return GRXBLAS_STATUS_EXECUTION_FAILED;
  if (n < 0) return GRXBLAS_STATUS_INVALID_VALUE;
  const size_t eb = elem_bytes(Btype), ec = elem_bytes(Ctype);
  if (eb == 0 || ec == 0) return GRXBLAS_STATUS_NOT_SUPPORTED;
  int start = 0, count = 0;
  grxblasShardRange(n, comm->rank, comm->world, &start, &count);
  const bool tb = transb == GRXBLAS_OP_T;
  // op(B) column j: stored column j (OP_N) or stored row j (OP_T)
  const void* Bj = B ? static_cast<const char*>(B) + (size_t)start * (tb ? 1 : (size_t)ldb) * eb : nullptr;
  void* Cj = C ? static_cast<char*>(C) + (size_t)start * (size_t)ldc * ec : nullptr;
  grxblasStatus_t st = GRXBLAS_STATUS_SUCCESS;
  if (count > 0 || n == 0) {
    st = grx::gemm_ex_columns(handle, transa, transb, m, count, k, alpha, A, Atype, lda, Bj, Btype, ldb, beta, Cj,
                              Ctype, ldc, start);
  } else if (!alpha || !beta || m < 0 || k < 0) {
    st = GRXBLAS_STATUS_INVALID_VALUE;  // a rank with no columns still validates like the others
  }
  if (st != GRXBLAS_STATUS_SUCCESS || !replicate || comm->world == 1 || m == 0 || n == 0) return st;

  // Replicated output: rank r's column block [start_r, start_r + count_r) of C
  // (count_r * ldc elements, ld padding rows included) is broadcast from r.
  const NcclApi* nc = nccl();
  cudaStream_t stream = nullptr;
  if (grxblasGetStream(handle, reinterpret_cast<grxStream_t*>(&stream)) != GRXBLAS_STATUS_SUCCESS)
    return GRXBLAS_STATUS_NOT_INITIALIZED;
  const double t0 = now_ms();
  ncclResult_t r = nc->GroupStart();
  for (int root = 0; root < comm->world && (r == ncclSuccess || r == ncclInProgress); ++root) {
    int s0 = 0, c0 = 0;
    grxblasShardRange(n, root, comm->world, &s0, &c0);
    if (c0 == 0) continue;
    char* blk = static_cast<char*>(C) + (size_t)s0 * (size_t)ldc * ec;
    r = nc->Broadcast(blk, blk, (size_t)c0 * (size_t)ldc * ec, ncclChar, root, comm->comm, stream);
  }
  const ncclResult_t e = nc->GroupEnd();
  if (r == ncclSuccess || r == ncclInProgress) r = e;
  if (r == ncclSuccess) {
    ncclResult_t a = ncclSuccess;
    if (nc->CommGetAsyncError(comm->comm, &a) != ncclSuccess) a = ncclInternalError;
    r = a;
  }
  return settle(*comm, r, t0);
}

grxblasStatus_t grxblasShardSynchronize(grxblasHandle_t handle, grxblasShardComm_t comm) {
  if (!handle) return GRXBLAS_STATUS_NOT_INITIALIZED;
  if (!comm) return GRXBLAS_STATUS_INVALID_VALUE;
  if (comm->broken) return GRXBLAS_STATUS_EXECUTION_FAILED;
  cudaStream_t stream = nullptr;
  if (grxblasGetStream(handle, reinterpret_cast<grxStream_t*>(&stream)) != GRXBLAS_STATUS_SUCCESS)
    return GRXBLAS_STATUS_NOT_INITIALIZED;
  const NcclApi* n = nccl();
  const double t0 = now_ms();
  for (;;) {
    const cudaError_t q = cudaStreamQuery(stream);
    if (q == cudaSuccess) break;
    if (q != cudaErrorNotReady) {
      cudaGetLastError();
      return GRXBLAS_STATUS_EXECUTION_FAILED;
    }
    ncclResult_t a = ncclSuccess;
    if (n->CommGetAsyncError(comm->comm, &a) != ncclSuccess) a = ncclInternalError;
    if ((a != ncclSuccess && a != ncclInProgress) || now_ms() - t0 > (double)deadline_ms()) {
      // a peer is gone: abort (this also ends the stuck NCCL kernels), then
      // let the stream drain
      n->CommAbort(comm->comm);
      comm->comm = nullptr;
      comm->broken = true;
      cudaStreamSynchronize(stream);
      cudaGetLastError();
      return GRXBLAS_STATUS_EXECUTION_FAILED;
    }
    nap();
  }
  return grxblasGetExecutionStatus(handle);
}

}  // extern "C"
