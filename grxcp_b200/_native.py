"""ctypes binding of libgrxcp.so: the C-ABI declared in include/grx/*.h.

This module only loads the library and declares prototypes; it never computes
anything itself. If the library is missing the import fails loudly -- there is
no CPU or PyTorch fallback anywhere in this package.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

LIB_PATH = Path(os.environ.get("GRXCP_LIB", Path(__file__).resolve().parent / "libgrxcp.so"))

if not LIB_PATH.exists():
    raise ImportError(
        f"grxcp_b200: native library not found at {LIB_PATH}; build it with "
        "`python -m grxcp_b200.build` (nvcc, sm_100a). There is no fallback path."
    )

lib = C.CDLL(str(LIB_PATH))

vp = C.c_void_p
i32 = C.c_int
i64 = C.c_longlong
f32 = C.c_float
u32 = C.c_uint
sz = C.c_size_t
fp = C.POINTER(C.c_float)
cp = C.c_char_p


class grxCycleSlot(C.Structure):
    _fields_ = [("start", C.c_uint64), ("end", C.c_uint64), ("core", C.c_uint32), ("warp", C.c_uint32)]


class grxblasEpilogue_t(C.Structure):
    _fields_ = [
        ("bias", vp),
        ("biasType", i32),
        ("strideBias", i64),
        ("scaleMode", i32),
        ("scaleA", vp),
        ("scaleB", vp),
        ("strideScaleA", i64),
        ("strideScaleB", i64),
        ("biasOverRows", i32),
        ("activation", i32),
    ]


class grxIpcMemHandle_t(C.Structure):
    _fields_ = [("reserved", C.c_ubyte * 64)]


class grxdnnConvDesc_t(C.Structure):
    _fields_ = [(f, i32) for f in ("n", "h", "w", "c", "k", "r", "s", "padH", "padW", "strideH", "strideW",
                                   "dilationH", "dilationW")]


class grxdnnPoolDesc_t(C.Structure):
    _fields_ = [(f, i32) for f in ("n", "h", "w", "c", "r", "s", "padH", "padW", "strideH", "strideW", "mode")]


class grxdnnAttnTensor_t(C.Structure):
    _fields_ = [
        ("batch", i32),
        ("heads", i32),
        ("seq", i32),
        ("headDim", i32),
        ("strideBatch", i64),
        ("strideHead", i64),
        ("strideSeq", i64),
        ("dtype", i32),
    ]


class grxDeviceProp_t(C.Structure):
    _fields_ = [
        ("name", C.c_char * 128),
        ("deviceType", i32),
        ("backend", i32),
        ("capabilities", u32),
        ("computeCapabilityMajor", i32),
        ("computeCapabilityMinor", i32),
        ("warpSize", i32),
        ("maxWarpsPerMultiProcessor", i32),
        ("multiProcessorCount", i32),
        ("clusterCount", i32),
        ("socketSize", i32),
        ("issueWidth", i32),
        ("maxThreadsPerBlock", i32),
        ("maxThreadsDim", i32 * 3),
        ("maxGridSize", i32 * 3),
        ("numBarriers", i32),
        ("totalGlobalMem", sz),
        ("sharedMemPerMultiprocessor", sz),
        ("sharedMemPerBlock", sz),
        ("memBankCount", i32),
        ("memBankSize", sz),
        ("cacheLineSize", i32),
        ("clockRateMHz", i32),
        ("peakMemoryBandwidthMBs", sz),
        ("unifiedAddressing", i32),
        ("managedMemory", i32),
        ("pinnedMemTotal", sz),
        ("pinnedMemFree", sz),
        ("warpShuffleIsEmulated", i32),
        ("eventTimingIsDeviceSide", i32),
        ("constantMemoryIsGlobal", i32),
    ]


# name -> (restype, argtypes). Every symbol of include/grx/*.h is listed here;
# tests check the two lists agree and that the library exports each one.
PROTOTYPES: dict[str, tuple] = {
    # grx_types.h / grx_runtime.h
    "grxGetErrorName": (cp, [i32]),
    "grxGetErrorString": (cp, [i32]),
    "grxGetDeviceCount": (i32, [C.POINTER(i32)]),
    "grxSetDevice": (i32, [i32]),
    "grxGetDevice": (i32, [C.POINTER(i32)]),
    "grxGetDeviceProperties": (i32, [C.POINTER(grxDeviceProp_t), i32]),
    "grxDeviceSynchronize": (i32, []),
    "grxMemGetInfo": (i32, [C.POINTER(sz), C.POINTER(sz)]),
    "grxDeviceCanAccessPeer": (i32, [C.POINTER(i32), i32, i32]),
    "grxDeviceEnablePeerAccess": (i32, [i32, u32]),
    "grxGetLastError": (i32, []),
    "grxPeekAtLastError": (i32, []),
    "grxMalloc": (i32, [C.POINTER(vp), sz]),
    "grxFree": (i32, [vp]),
    "grxMallocHost": (i32, [C.POINTER(vp), sz]),
    "grxFreeHost": (i32, [vp]),
    "grxMemcpy": (i32, [vp, vp, sz, i32]),
    "grxMemcpyAsync": (i32, [vp, vp, sz, i32, vp]),
    "grxMemset": (i32, [vp, i32, sz]),
    "grxMemsetAsync": (i32, [vp, i32, sz, vp]),
    "grxStreamCreate": (i32, [C.POINTER(vp)]),
    "grxStreamCreateWithFlags": (i32, [C.POINTER(vp), u32]),
    "grxStreamDestroy": (i32, [vp]),
    "grxStreamSynchronize": (i32, [vp]),
    "grxStreamQuery": (i32, [vp]),
    "grxStreamWaitEvent": (i32, [vp, vp, u32]),
    "grxEventCreate": (i32, [C.POINTER(vp)]),
    "grxEventCreateWithFlags": (i32, [C.POINTER(vp), u32]),
    "grxEventDestroy": (i32, [vp]),
    "grxEventRecord": (i32, [vp, vp]),
    "grxEventSynchronize": (i32, [vp]),
    "grxEventQuery": (i32, [vp]),
    "grxEventElapsedTime": (i32, [fp, vp, vp]),
    # grx_tensormap.h (the desc argument is passed as an opaque pointer)
    "grxTensorMapGetSlotCount": (i32, [C.POINTER(i32), i32]),
    "grxMallocPhysical": (i32, [C.POINTER(vp), sz]),
    "grxTensorMapProgramAsync": (i32, [vp, vp]),
    "grxTensorMapProgram": (i32, [vp]),
    # grxblas.h
    "grxblasGetStatusString": (cp, [i32]),
    "grxblasCreate": (i32, [C.POINTER(vp)]),
    "grxblasDestroy": (i32, [vp]),
    "grxblasSetStream": (i32, [vp, vp]),
    "grxblasGetStream": (i32, [vp, C.POINTER(vp)]),
    "grxblasGemmEx": (i32, [vp, i32, i32, i32, i32, i32, fp, vp, i32, i32, vp, i32, i32, fp, vp, i32, i32]),
    "grxblasGemmStridedBatchedEx": (
        i32,
        [vp, i32, i32, i32, i32, i32, fp, vp, i32, i32, i64, vp, i32, i32, i64, fp, vp, i32, i32, i64, i32],
    ),
    "grxblasSetEpilogue": (i32, [vp, C.POINTER(grxblasEpilogue_t)]),
    "grxblasGetTensorTypes": (i32, [vp, C.POINTER(u32)]),
    "grxblasSetTensorMapSlots": (i32, [vp, i32, i32]),
    "grxblasGetTensorTile": (i32, [vp, C.POINTER(i32), C.POINTER(i32), C.POINTER(i32)]),
    "grxblasSaxpy": (i32, [vp, i32, fp, vp, i32, vp, i32]),
    "grxblasSscal": (i32, [vp, i32, fp, vp, i32]),
    "grxblasSgemv": (i32, [vp, i32, i32, i32, fp, vp, i32, vp, i32, fp, vp, i32]),
    "grxblasSgemm": (i32, [vp, i32, i32, i32, i32, i32, fp, vp, i32, vp, i32, fp, vp, i32]),
    "grxblasSgemmStridedBatched": (
        i32,
        [vp, i32, i32, i32, i32, i32, fp, vp, i32, i64, vp, i32, i64, fp, vp, i32, i64, i32],
    ),
    "grxblasSetKernelPath": (i32, [cp]),
    "grxblasSetCycleProbe": (i32, [vp, vp, i32]),
    "grxblasCycleSlotsNeeded": (i32, [vp, i32, i32]),
    "grxblasGetLoadedKernelPath": (i32, [vp, C.POINTER(cp)]),
    "grxblasSetWorkspace": (i32, [vp, vp, sz]),
    "grxblasGetWorkspaceSize": (sz, [vp, i32, i32, i32, i32, i32, i32, i32, i32, i32, i32]),
    "grxblasGetExecutionStatus": (i32, [vp]),
    "grxblasShardGetUniqueId": (i32, [vp]),
    "grxblasShardCommInit": (i32, [C.POINTER(vp), vp, i32, i32]),
    "grxblasShardCommDestroy": (i32, [vp]),
    "grxblasShardRange": (i32, [i32, i32, i32, C.POINTER(i32), C.POINTER(i32)]),
    "grxblasGemmExColumnParallel": (i32, [vp, vp, i32, i32, i32, i32, i32, fp, vp, i32, i32, vp, i32, i32, fp, vp,
                                          i32, i32, i32]),
    "grxblasShardSynchronize": (i32, [vp, vp]),
    "grxblasGemmExNoAlloc": (i32, [vp, i32, i32, i32, i32, i32, fp, vp, i32, i32, vp, i32, i32, fp, vp, i32, i32, vp]),
    # grxdnn.h
    "grxdnnGetStatusString": (cp, [i32]),
    "grxdnnCreate": (i32, [C.POINTER(vp)]),
    "grxdnnDestroy": (i32, [vp]),
    "grxdnnSetStream": (i32, [vp, vp]),
    "grxdnnGetStream": (i32, [vp, C.POINTER(vp)]),
    "grxdnnRMSNormForward": (i32, [vp, i32, i32, vp, i32, i64, vp, f32, vp, i32, i64, vp]),
    "grxdnnLayerNormForward": (i32, [vp, i32, i32, vp, i32, i64, vp, vp, f32, vp, i32, i64, vp, vp]),
    "grxdnnRMSNormBackward": (i32, [vp, i32, i32, vp, i32, i64, vp, i32, i64, vp, vp, f32, vp, i32, i64, vp]),
    "grxdnnLayerNormBackward": (i32, [vp, i32, i32, vp, i32, i64, vp, i32, i64, vp, vp, vp, f32, vp, i32, i64, vp, vp]),
    "grxdnnAttentionForward": (
        i32,
        [
            vp,
            C.POINTER(grxdnnAttnTensor_t),
            vp,
            C.POINTER(grxdnnAttnTensor_t),
            vp,
            C.POINTER(grxdnnAttnTensor_t),
            vp,
            C.POINTER(grxdnnAttnTensor_t),
            vp,
            f32,
            i32,
            vp,
        ],
    ),
    "grxblasSetPeerOutputs": (i32, [vp, i32, vp]),
    "grxIpcGetMemHandle": (i32, [vp, vp]),
    "grxIpcOpenMemHandle": (i32, [vp, grxIpcMemHandle_t]),
    "grxIpcCloseMemHandle": (i32, [vp]),
    "grxdnnSoftmaxBackward": (i32, [vp, i32, i32, vp, i32, i64, vp, i32, i64, vp, i32, i64]),
    "grxdnnGeluBackward": (i32, [vp, i64, vp, vp, vp, i32, i32]),
    "grxdnnConvOutputDims": (i32, [vp, vp, vp]),
    "grxdnnConv2dForward": (i32, [vp, vp, vp, i32, vp, i32, vp, vp, vp, i32, vp, i32]),
    "grxdnnPoolingOutputDims": (i32, [vp, vp, vp]),
    "grxdnnPooling2dForward": (i32, [vp, vp, vp, i32, vp, i32]),
    "grxdnnAttentionBackward": (i32, [vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, f32, i32, vp, vp, vp, vp, vp, vp]),
    "grxdnnGetExecutionStatus": (i32, [vp]),
    "grxdnnSoftmaxForward": (i32, [vp, i32, i32, vp, i32, i64, vp, i32, i64]),
    "grxdnnGeluForward": (i32, [vp, i64, vp, i32, vp, i32, i32]),
}

# Internal test hook (not in the public headers).
INTERNAL = {"grxcpTestBoundedWait": (i32, [C.c_ulonglong])}

for _name, (_res, _args) in {**PROTOTYPES, **INTERNAL}.items():
    _f = getattr(lib, _name)
    _f.restype = _res
    _f.argtypes = _args

# Element type and status codes (include/grx/grx_types.h, grxblas.h).
GRX_R_32F, GRX_R_16F, GRX_R_8I, GRX_R_32I, GRX_R_16BF, GRX_R_8F_E4M3 = 0, 2, 3, 10, 14, 28
OP_N, OP_T = 0, 1
STATUS = {
    0: "SUCCESS",
    1: "NOT_INITIALIZED",
    2: "ALLOC_FAILED",
    3: "INVALID_VALUE",
    4: "ARCH_MISMATCH",
    5: "EXECUTION_FAILED",
    6: "NOT_SUPPORTED",
    7: "INTERNAL_ERROR",
}
SUCCESS, NOT_INITIALIZED, ALLOC_FAILED, INVALID_VALUE, ARCH_MISMATCH, EXECUTION_FAILED, NOT_SUPPORTED, INTERNAL_ERROR = range(8)
SCALE_NONE, SCALE_TENSOR, SCALE_ROWCOL = 0, 1, 2
ACT_NONE, ACT_RELU, ACT_GELU_TANH, ACT_GELU_ERF = 0, 1, 2, 3

POOL_MAX, POOL_AVG_INCLUDE_PAD, POOL_AVG_EXCLUDE_PAD = 0, 1, 2
