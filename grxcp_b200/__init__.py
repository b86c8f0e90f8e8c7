"""grxcp_b200 -- the GRXCP math-library hot path (grxBLAS GEMM, grxDNN
attention / RMSNorm / LayerNorm) rebuilt for NVIDIA B200 (sm_100a).

The product is the C-ABI shared library ``libgrxcp.so`` (headers under
``include/grx``); this package loads it and mirrors its entry points:

    grxcp_b200.blas    grxblas* (handle, GemmEx, Sgemm, strided batched, L1/L2)
    grxcp_b200.dnn     grxdnn*  (RMSNorm, LayerNorm, attention forward)
    grxcp_b200.shard   column-parallel GEMM / (batch x head)-parallel attention
                       over torch.distributed ranks, optional NCCL all-gather
"""
from . import _native, blas, dnn  # noqa: F401

__all__ = ["blas", "dnn", "_native"]
