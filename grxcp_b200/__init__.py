"""grxcp_b200 -- the GRXCP math-library hot path (grxBLAS GEMM, grxDNN
attention / RMSNorm / LayerNorm) rebuilt for NVIDIA B200 (sm_100a).

The product is the C-ABI shared library ``libgrxcp.so`` (headers under
``include/grx``); this package loads it and mirrors its entry points:

    grxcp_b200.blas    grxblas* (handle, GemmEx, Sgemm, strided batched, L1/L2)
    grxcp_b200.dnn     grxdnn*  (RMSNorm, LayerNorm, attention forward)
    grxcp_b200.shard   column-parallel GEMM / (batch x head)-parallel attention
                       over torch.distributed ranks, optional NCCL all-gather

Submodules load on first use, so ``python -m grxcp_b200.build`` works before
the library exists.
"""
import importlib

__all__ = ["blas", "dnn", "shard", "_native"]


def __getattr__(name):
    if name in __all__:
        return importlib.import_module(f"{__name__}.{name}")
    raise AttributeError(name)
