"""grxBLAS from Python: the reference's grxblas* C API, one method per entry point.

Method names, argument order and meaning are those of include/grx/grxblas.h
(reference: kubeworkz/grxcp include/grx/grxblas.h:53-248). Every method calls
the C-ABI of libgrxcp.so and returns its raw status code, exactly as a C
caller would see it; ``check()`` turns a non-success status into an exception.
Matrix arguments may be torch tensors (their data pointer is passed) or plain
integer device addresses.
"""
from __future__ import annotations

import ctypes as C

from . import _native as N
from ._native import lib


class GrxblasError(RuntimeError):
    def __init__(self, status: int, what: str = ""):
        self.status = status
        msg = lib.grxblasGetStatusString(status).decode()
        super().__init__(f"{what}: {N.STATUS.get(status, status)} ({msg})")


def check(status: int, what: str = "grxblas") -> None:
    if status != N.SUCCESS:
        raise GrxblasError(status, what)


def ptr(x) -> int | None:
    """Device address of a tensor (or an int passed through); None -> NULL."""
    if x is None:
        return None
    if isinstance(x, int):
        return x
    return x.data_ptr()


def dtype_code(t) -> int:
    import torch

    table = {
        torch.float32: N.GRX_R_32F,
        torch.float16: N.GRX_R_16F,
        torch.bfloat16: N.GRX_R_16BF,
        torch.int8: N.GRX_R_8I,
        torch.int32: N.GRX_R_32I,
        torch.float8_e4m3fn: N.GRX_R_8F_E4M3,
    }
    return table[t.dtype if hasattr(t, "dtype") else t]


def _fptr(v: float | None):
    return None if v is None else C.byref(C.c_float(v))


def stream_ptr(stream) -> int | None:
    if stream is None:
        return None
    if isinstance(stream, int):
        return stream
    return stream.cuda_stream


class Handle:
    """A grxblasHandle_t (reference grxblas.cpp:426-450)."""

    def __init__(self):
        h = C.c_void_p()
        check(lib.grxblasCreate(C.byref(h)), "grxblasCreate")
        self.h = h

    def close(self) -> int:
        if self.h:
            s = lib.grxblasDestroy(self.h)
            self.h = None
            return s
        return N.SUCCESS

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # -- handle state
    def set_stream(self, stream) -> int:
        return lib.grxblasSetStream(self.h, stream_ptr(stream))

    def get_stream(self) -> int:
        s = C.c_void_p()
        check(lib.grxblasGetStream(self.h, C.byref(s)))
        return s.value or 0

    def set_epilogue(self, bias=None, bias_type=None, stride_bias=0, scale_mode=N.SCALE_NONE, scale_a=None,
                     scale_b=None, stride_scale_a=0, stride_scale_b=0, bias_over_rows=False,
                     activation=N.ACT_NONE) -> int:
        e = N.grxblasEpilogue_t()
        e.bias = ptr(bias)
        e.biasType = bias_type if bias_type is not None else (dtype_code(bias) if bias is not None else N.GRX_R_32F)
        e.strideBias = stride_bias
        e.scaleMode = scale_mode
        e.scaleA = ptr(scale_a)
        e.scaleB = ptr(scale_b)
        e.strideScaleA = stride_scale_a
        e.strideScaleB = stride_scale_b
        e.biasOverRows = 1 if bias_over_rows else 0
        e.activation = activation
        return lib.grxblasSetEpilogue(self.h, C.byref(e))

    def clear_epilogue(self) -> int:
        return lib.grxblasSetEpilogue(self.h, None)

    def set_peer_outputs(self, peers) -> int:
        """grxblasSetPeerOutputs: device addresses (ints) of peer copies of C; [] clears."""
        arr = (C.c_void_p * max(1, len(peers)))(*[C.c_void_p(int(x)) for x in peers])
        return lib.grxblasSetPeerOutputs(self.h, len(peers), arr if peers else None)

    def set_workspace(self, ws, nbytes: int) -> int:
        return lib.grxblasSetWorkspace(self.h, ptr(ws), nbytes)

    def tensor_types(self) -> tuple[int, int]:
        m = C.c_uint()
        s = lib.grxblasGetTensorTypes(self.h, C.byref(m))
        return s, m.value

    def tensor_tile(self) -> tuple[int, tuple[int, int, int]]:
        a, b, c = C.c_int(), C.c_int(), C.c_int()
        s = lib.grxblasGetTensorTile(self.h, C.byref(a), C.byref(b), C.byref(c))
        return s, (a.value, b.value, c.value)

    def set_tensor_map_slots(self, a: int, b: int) -> int:
        return lib.grxblasSetTensorMapSlots(self.h, a, b)

    def execution_status(self) -> int:
        return lib.grxblasGetExecutionStatus(self.h)

    def loaded_kernel_path(self) -> str | None:
        p = C.c_char_p()
        check(lib.grxblasGetLoadedKernelPath(self.h, C.byref(p)))
        return p.value.decode() if p.value else None

    def set_cycle_probe(self, slots, capacity: int) -> int:
        return lib.grxblasSetCycleProbe(self.h, ptr(slots), capacity)

    # -- GEMM
    def gemm_ex(self, transa, transb, m, n, k, alpha, A, Atype, lda, B, Btype, ldb, beta, C_, Ctype, ldc) -> int:
        return lib.grxblasGemmEx(self.h, transa, transb, m, n, k, _fptr(alpha), ptr(A), Atype, lda, ptr(B), Btype,
                                 ldb, _fptr(beta), ptr(C_), Ctype, ldc)

    def gemm_strided_batched_ex(self, transa, transb, m, n, k, alpha, A, Atype, lda, sA, B, Btype, ldb, sB, beta,
                                C_, Ctype, ldc, sC, batch) -> int:
        return lib.grxblasGemmStridedBatchedEx(self.h, transa, transb, m, n, k, _fptr(alpha), ptr(A), Atype, lda, sA,
                                               ptr(B), Btype, ldb, sB, _fptr(beta), ptr(C_), Ctype, ldc, sC, batch)

    def sgemm(self, transa, transb, m, n, k, alpha, A, lda, B, ldb, beta, C_, ldc) -> int:
        return lib.grxblasSgemm(self.h, transa, transb, m, n, k, _fptr(alpha), ptr(A), lda, ptr(B), ldb, _fptr(beta),
                                ptr(C_), ldc)

    def sgemm_strided_batched(self, transa, transb, m, n, k, alpha, A, lda, sA, B, ldb, sB, beta, C_, ldc, sC,
                              batch) -> int:
        return lib.grxblasSgemmStridedBatched(self.h, transa, transb, m, n, k, _fptr(alpha), ptr(A), lda, sA, ptr(B),
                                              ldb, sB, _fptr(beta), ptr(C_), ldc, sC, batch)

    # -- level 1 / 2
    def saxpy(self, n, alpha, x, incx, y, incy) -> int:
        return lib.grxblasSaxpy(self.h, n, _fptr(alpha), ptr(x), incx, ptr(y), incy)

    def sscal(self, n, alpha, x, incx) -> int:
        return lib.grxblasSscal(self.h, n, _fptr(alpha), ptr(x), incx)

    def sgemv(self, trans, m, n, alpha, A, lda, x, incx, beta, y, incy) -> int:
        return lib.grxblasSgemv(self.h, trans, m, n, _fptr(alpha), ptr(A), lda, ptr(x), incx, _fptr(beta), ptr(y),
                                incy)


def set_kernel_path(path: str | None) -> int:
    return lib.grxblasSetKernelPath(path.encode() if path is not None else None)


def cycle_slots_needed(m: int, n: int) -> int:
    return lib.grxblasCycleSlotsNeeded(None, m, n)


# ------------------------------------------------------------------ column-parallel over NCCL

def shard_unique_id() -> tuple[int, bytes]:
    """grxblasShardGetUniqueId: (status, the 128-byte id rank 0 hands to the others)."""
    buf = C.create_string_buffer(128)
    st = lib.grxblasShardGetUniqueId(buf)
    return st, buf.raw


def shard_range(n: int, rank: int, world: int) -> tuple[int, int, int]:
    """grxblasShardRange: (status, start, count)."""
    s, c = C.c_int(0), C.c_int(0)
    st = lib.grxblasShardRange(n, rank, world, C.byref(s), C.byref(c))
    return st, s.value, c.value


class ShardComm:
    """One rank's NCCL communicator for grxblasGemmExColumnParallel (current device)."""

    def __init__(self, uid: bytes, rank: int, world: int):
        self.c = C.c_void_p()
        self.rank, self.world = rank, world
        idbuf = C.create_string_buffer(uid, 128)
        self.status = lib.grxblasShardCommInit(C.byref(self.c), idbuf, rank, world)

    def destroy(self) -> int:
        st = N.SUCCESS
        if self.c:
            st = lib.grxblasShardCommDestroy(self.c)
            self.c = C.c_void_p()
        return st

    def gemm_ex_column_parallel(self, handle: "Handle", transa, transb, m, n, k, alpha, A, Atype, lda, B, Btype, ldb,
                                beta, C_, Ctype, ldc, replicate: bool) -> int:
        return lib.grxblasGemmExColumnParallel(handle.h, self.c, transa, transb, m, n, k, _fptr(alpha), ptr(A), Atype,
                                               lda, ptr(B), Btype, ldb, _fptr(beta), ptr(C_), Ctype, ldc,
                                               1 if replicate else 0)

    def synchronize(self, handle: "Handle") -> int:
        return lib.grxblasShardSynchronize(handle.h, self.c)
