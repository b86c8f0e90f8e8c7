"""grxDNN from Python: norms (forward and backward), softmax, GELU, conv2d, pooling and attention (forward and backward).

Thin mirror of include/grx/grxdnn.h; every method returns the raw status code
of the C call. Tensors are torch CUDA tensors (or integer device addresses).
"""
from __future__ import annotations

import ctypes as C

from . import _native as N
from ._native import lib
from .blas import dtype_code, ptr, stream_ptr


class GrxdnnError(RuntimeError):
    def __init__(self, status: int, what: str = ""):
        self.status = status
        super().__init__(f"{what}: {N.STATUS.get(status, status)} ({lib.grxdnnGetStatusString(status).decode()})")


def check(status: int, what: str = "grxdnn") -> None:
    if status != N.SUCCESS:
        raise GrxdnnError(status, what)


def attn_desc(t, batch=None, heads=None, seq=None, head_dim=None, dtype=None) -> N.grxdnnAttnTensor_t:
    """Descriptor of a [batch, heads, seq, head_dim] tensor (strides in elements)."""
    d = N.grxdnnAttnTensor_t()
    if t is not None and hasattr(t, "stride"):
        b, h, s, hd = t.shape
        sb, sh, ss, sd = t.stride()
        if sd != 1:
            raise ValueError("head_dim must be contiguous")
        d.batch, d.heads, d.seq, d.headDim = b, h, s, hd
        d.strideBatch, d.strideHead, d.strideSeq = sb, sh, ss
        d.dtype = dtype_code(t)
    else:
        d.batch, d.heads, d.seq, d.headDim = batch, heads, seq, head_dim
        d.strideBatch, d.strideHead, d.strideSeq = heads * seq * head_dim, seq * head_dim, head_dim
        d.dtype = dtype if dtype is not None else N.GRX_R_16BF
    return d


def conv_desc(x, w, pad=(0, 0), stride=(1, 1), dilation=(1, 1)):
    n, h, wd, c = x.shape
    k, r, s, _ = w.shape
    return N.grxdnnConvDesc_t(n, h, wd, c, k, r, s, pad[0], pad[1], stride[0], stride[1], dilation[0], dilation[1])


def conv_out_dims(d) -> tuple[int, int]:
    p, q = C.c_int(), C.c_int()
    st = lib.grxdnnConvOutputDims(C.byref(d), C.byref(p), C.byref(q))
    if st != 0:
        raise ValueError(f"bad conv geometry (status {st})")
    return p.value, q.value


def pool_desc(x, window, pad=(0, 0), stride=(1, 1), mode=0):
    n, h, wd, c = x.shape
    return N.grxdnnPoolDesc_t(n, h, wd, c, window[0], window[1], pad[0], pad[1], stride[0], stride[1], mode)


class Handle:
    def __init__(self):
        h = C.c_void_p()
        check(lib.grxdnnCreate(C.byref(h)), "grxdnnCreate")
        self.h = h

    def close(self) -> int:
        if self.h:
            s = lib.grxdnnDestroy(self.h)
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

    def set_stream(self, stream) -> int:
        return lib.grxdnnSetStream(self.h, stream_ptr(stream))

    def execution_status(self) -> int:
        return lib.grxdnnGetExecutionStatus(self.h)

    def rmsnorm(self, x, gamma, eps, y, rstd=None, rows=None, hidden=None, ldx=None, ldy=None) -> int:
        rows = x.shape[0] if rows is None else rows
        hidden = x.shape[1] if hidden is None else hidden
        ldx = x.stride(0) if ldx is None else ldx
        ldy = y.stride(0) if ldy is None else ldy
        return lib.grxdnnRMSNormForward(self.h, rows, hidden, ptr(x), dtype_code(x), ldx, ptr(gamma), eps, ptr(y),
                                        dtype_code(y), ldy, ptr(rstd))

    def layernorm(self, x, gamma, beta, eps, y, mean=None, rstd=None, rows=None, hidden=None, ldx=None,
                  ldy=None) -> int:
        rows = x.shape[0] if rows is None else rows
        hidden = x.shape[1] if hidden is None else hidden
        ldx = x.stride(0) if ldx is None else ldx
        ldy = y.stride(0) if ldy is None else ldy
        return lib.grxdnnLayerNormForward(self.h, rows, hidden, ptr(x), dtype_code(x), ldx, ptr(gamma), ptr(beta),
                                          eps, ptr(y), dtype_code(y), ldy, ptr(mean), ptr(rstd))

    def rmsnorm_backward(self, dy, x, gamma, eps, dx, rstd=None, dgamma=None) -> int:
        """grxdnnRMSNormBackward on [rows, hidden] tensors with row pitches from strides."""
        rows, hidden = x.shape
        return lib.grxdnnRMSNormBackward(self.h, rows, hidden, ptr(dy), dtype_code(dy), dy.stride(0), ptr(x),
                                         dtype_code(x), x.stride(0), ptr(gamma), ptr(rstd), eps, ptr(dx),
                                         dtype_code(dx), dx.stride(0), ptr(dgamma))

    def layernorm_backward(self, dy, x, gamma, eps, dx, mean=None, rstd=None, dgamma=None, dbeta=None) -> int:
        """grxdnnLayerNormBackward on [rows, hidden] tensors with row pitches from strides."""
        rows, hidden = x.shape
        return lib.grxdnnLayerNormBackward(self.h, rows, hidden, ptr(dy), dtype_code(dy), dy.stride(0), ptr(x),
                                           dtype_code(x), x.stride(0), ptr(gamma), ptr(mean), ptr(rstd), eps,
                                           ptr(dx), dtype_code(dx), dx.stride(0), ptr(dgamma), ptr(dbeta))

    def softmax(self, x, y, rows=None, cols=None, ldx=None, ldy=None) -> int:
        rows = x.shape[0] if rows is None else rows
        cols = x.shape[1] if cols is None else cols
        ldx = x.stride(0) if ldx is None else ldx
        ldy = y.stride(0) if ldy is None else ldy
        return lib.grxdnnSoftmaxForward(self.h, rows, cols, ptr(x), dtype_code(x), ldx, ptr(y), dtype_code(y), ldy)

    def gelu(self, x, y, mode: int = 0, n=None) -> int:
        n = x.numel() if n is None else n
        return lib.grxdnnGeluForward(self.h, n, ptr(x), dtype_code(x), ptr(y), dtype_code(y), mode)

    def attention_backward(self, q, k, v, o, dout, lse, scale, causal, dq, dk, dv) -> int:
        """grxdnnAttentionBackward on [B, H, S, D] tensors (descriptors from strides)."""
        ds = [attn_desc(t) for t in (q, k, v, o, dout, dq, dk, dv)]
        return lib.grxdnnAttentionBackward(self.h, C.byref(ds[0]), ptr(q), C.byref(ds[1]), ptr(k), C.byref(ds[2]),
                                           ptr(v), C.byref(ds[3]), ptr(o), C.byref(ds[4]), ptr(dout), ptr(lse),
                                           scale, 1 if causal else 0, C.byref(ds[5]), ptr(dq), C.byref(ds[6]),
                                           ptr(dk), C.byref(ds[7]), ptr(dv))

    def conv2d(self, x, w, y, pad=(0, 0), stride=(1, 1), dilation=(1, 1), bias=None, activation=0, alpha=None,
               beta=None) -> int:
        """grxdnnConv2dForward: x [n, h, w, c] NHWC, w [k, r, s, c] KRSC, y [n, p, q, k]."""
        d = conv_desc(x, w, pad, stride, dilation)
        a = C.c_float(alpha) if alpha is not None else None
        b = C.c_float(beta) if beta is not None else None
        return lib.grxdnnConv2dForward(self.h, C.byref(d), ptr(x), dtype_code(x), ptr(w), dtype_code(w),
                                       C.byref(a) if a is not None else None, C.byref(b) if b is not None else None,
                                       ptr(bias), activation, ptr(y), dtype_code(y))

    def pool2d(self, x, y, window, pad=(0, 0), stride=None, mode=0) -> int:
        """grxdnnPooling2dForward on NHWC tensors."""
        d = pool_desc(x, window, pad, stride or window, mode)
        return lib.grxdnnPooling2dForward(self.h, C.byref(d), ptr(x), dtype_code(x), ptr(y), dtype_code(y))

    def softmax_backward(self, y, dy, dx) -> int:
        """grxdnnSoftmaxBackward on [rows, cols] tensors (row pitches from strides)."""
        rows, cols = y.shape
        return lib.grxdnnSoftmaxBackward(self.h, rows, cols, ptr(y), dtype_code(y), y.stride(0), ptr(dy),
                                         dtype_code(dy), dy.stride(0), ptr(dx), dtype_code(dx), dx.stride(0))

    def gelu_backward(self, x, dy, dx, mode: int = 0) -> int:
        """grxdnnGeluBackward over x.numel() contiguous elements."""
        return lib.grxdnnGeluBackward(self.h, x.numel(), ptr(x), ptr(dy), ptr(dx), dtype_code(x), mode)

    def attention(self, q, k, v, o, scale, causal, lse=None, descs=None) -> int:
        dq, dk, dv, do = descs if descs is not None else (attn_desc(q), attn_desc(k), attn_desc(v), attn_desc(o))
        return lib.grxdnnAttentionForward(self.h, C.byref(dq), ptr(q), C.byref(dk), ptr(k), C.byref(dv), ptr(v),
                                          C.byref(do), ptr(o), scale, 1 if causal else 0, ptr(lse))
