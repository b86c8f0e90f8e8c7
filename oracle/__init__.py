"""CPU oracle for grxcp-b200 -- TEST INFRASTRUCTURE, never the product path.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs import
this package, and only as the checker (or as the timed CPU baseline). It wraps
``liboracle.so`` (oracle.c, plain gcc) with numpy; see oracle.c for the
reference file:line each function restates.

Parity status: the GEMM gates (fp32 sgemm, fp16 exact GemmEx, int8 -> int32)
are pinned by the reference's own test-gate loops and known-answer tests, and
the fp32 sgemm kernel is additionally pinned against the reference's sgemm
kernel source compiled for the host (oracle/_ref, built by build_ref.py). bf16
/ fp8 / scaled-int8 GEMM, RMSNorm, LayerNorm and attention have no code in the
reference: for those the oracle is the fp64 definition, parity unpinned by the
reference itself.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "liboracle.so"


def build(force: bool = False) -> Path:
    src = HERE / "oracle.c"
    if force or not LIB_PATH.exists() or LIB_PATH.stat().st_mtime < src.stat().st_mtime:
        cmd = ["gcc", "-O2", "-std=c11", "-fPIC", "-shared", "-ffp-contract=off", "-fno-fast-math", "-o",
               str(LIB_PATH), str(src), "-lm", "-lpthread"]
        subprocess.run(cmd, check=True)
    return LIB_PATH


build()
_lib = C.CDLL(str(LIB_PATH))

_vp = C.c_void_p
_i = C.c_int
_ll = C.c_longlong
_f = C.c_float
_d = C.c_double

_protos = {
    "ora_f32_to_bf16": (C.c_uint16, [_f]),
    "ora_bf16_to_f32": (_f, [C.c_uint16]),
    "ora_f32_to_f16": (C.c_uint16, [_f]),
    "ora_f16_to_f32": (_f, [C.c_uint16]),
    "ora_f32_to_e4m3": (C.c_uint8, [_f]),
    "ora_e4m3_to_f32": (_f, [C.c_uint8]),
    "ora_encode": (None, [_i, _vp, _vp, _ll]),
    "ora_decode": (None, [_i, _vp, _vp, _ll]),
    "ora_sgemm_ref": (None, [_i, _i, _i, _i, _i, _f, _vp, _i, _vp, _i, _f, _vp, _i]),
    "ora_sgemm_kernel": (None, [_i, _i, _i, _i, _i, _f, _vp, _i, _ll, _vp, _i, _ll, _f, _vp, _i, _ll, _i]),
    "ora_gemm_f32seq": (None, [_i, _i, _i, _i, _i, _f, _vp, _i, _vp, _i, _f, _vp, _i]),
    "ora_igemm": (None, [_i, _i, _i, _i, _i, _i, _vp, _i, _vp, _i, _i, _vp, _i]),
    "ora_igemm_npu": (None, [_i, _i, _i, _i, _i, _vp, _i, _vp, _i, _vp, _i]),
    "ora_gemm_f64": (
        None,
        [_i, _i, _i, _i, _i, _d, _vp, _i, _ll, _vp, _i, _ll, _d, _vp, _vp, _i, _ll, _i, _vp, _ll, _i, _vp, _vp, _ll,
         _ll, _i, _i, _i],
    ),
    "ora_rmsnorm": (None, [_i, _i, _vp, _ll, _vp, _d, _vp, _vp, _i]),
    "ora_norm_bwd": (None, [_i, _i, _i, _vp, _vp, _vp, _d, _vp, _vp, _vp]),
    "ora_layernorm": (None, [_i, _i, _vp, _ll, _vp, _vp, _d, _vp, _vp, _vp, _i]),
    "ora_attention": (None, [_i, _i, _i, _i, _vp, _vp, _vp, _d, _i, _vp, _i, _i, _i, _vp, _vp, _i]),
    "ora_conv2d": (None, [_i] * 15 + [_vp, _vp, _vp]),
    "ora_attention_bwd": (None, [_i, _i, _i, _i, _vp, _vp, _vp, _vp, _d, _i, _vp, _vp, _vp, _i]),
    "ora_saxpy": (None, [_i, _f, _vp, _i, _vp, _i]),
    "ora_softmax": (None, [_i, _i, _vp, _ll, _vp]),
    "ora_gelu": (None, [_ll, _vp, _vp, _i]),
    "ora_sscal": (None, [_i, _f, _vp, _i]),
    "ora_sgemv": (None, [_i, _i, _i, _f, _vp, _i, _vp, _i, _f, _vp, _i]),
}
for _n, (_r, _a) in _protos.items():
    getattr(_lib, _n).restype = _r
    getattr(_lib, _n).argtypes = _a

KIND = {"bf16": 0, "f16": 1, "e4m3": 2}


def _p(a: np.ndarray | None):
    return None if a is None else a.ctypes.data_as(_vp)


def nthreads_default() -> int:
    return max(1, len(os.sched_getaffinity(0)))


# ------------------------------------------------------------ conversions

def encode(kind: str, x) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, dtype=np.uint8 if kind == "e4m3" else np.uint16)
    _lib.ora_encode(KIND[kind], _p(x), _p(out), x.size)
    return out


def decode(kind: str, bits) -> np.ndarray:
    bits = np.ascontiguousarray(bits)
    out = np.empty(bits.shape, dtype=np.float32)
    _lib.ora_decode(KIND[kind], _p(bits), _p(out), bits.size)
    return out


def round_to(kind: str, x) -> np.ndarray:
    """Values of x after rounding to `kind` (RNE; e4m3 saturating)."""
    return decode(kind, encode(kind, x))


# ------------------------------------------------------------ GEMM

def sgemm_ref(ta, tb, m, n, k, alpha, A, lda, B, ldb, beta, Cbuf, ldc) -> np.ndarray:
    """tests/libs/test_grxblas.cpp:63-80 on column-major float buffers; returns a new C buffer."""
    A = np.ascontiguousarray(A, np.float32)
    B = np.ascontiguousarray(B, np.float32)
    out = np.array(Cbuf, dtype=np.float32, copy=True)
    _lib.ora_sgemm_ref(int(ta), int(tb), m, n, k, alpha, _p(A), lda, _p(B), ldb, beta, _p(out), ldc)
    return out


def sgemm_kernel(ta, tb, m, n, k, alpha, A, lda, sA, B, ldb, sB, beta, Cbuf, ldc, sC, batch) -> np.ndarray:
    A = np.ascontiguousarray(A, np.float32)
    B = np.ascontiguousarray(B, np.float32)
    out = np.array(Cbuf, dtype=np.float32, copy=True)
    _lib.ora_sgemm_kernel(int(ta), int(tb), m, n, k, alpha, _p(A), lda, sA, _p(B), ldb, sB, beta, _p(out), ldc, sC,
                          batch)
    return out


def gemm_f32seq(ta, tb, m, n, k, alpha, A, lda, B, ldb, beta, Cbuf, ldc) -> np.ndarray:
    A = np.ascontiguousarray(A, np.float32)
    B = np.ascontiguousarray(B, np.float32)
    out = np.array(Cbuf, dtype=np.float32, copy=True)
    _lib.ora_gemm_f32seq(int(ta), int(tb), m, n, k, alpha, _p(A), lda, _p(B), ldb, beta, _p(out), ldc)
    return out


def igemm(ta, tb, m, n, k, alpha, A, lda, B, ldb, beta, Cbuf, ldc) -> np.ndarray:
    A = np.ascontiguousarray(A, np.int8)
    B = np.ascontiguousarray(B, np.int8)
    out = np.array(Cbuf, dtype=np.int32, copy=True)
    _lib.ora_igemm(int(ta), int(tb), m, n, k, int(alpha), _p(A), lda, _p(B), ldb, int(beta), _p(out), ldc)
    return out


def igemm_npu(m, n, k, alpha, beta, A, lda, B, ldb, Cbuf, ldc) -> np.ndarray:
    A = np.ascontiguousarray(A, np.int8)
    B = np.ascontiguousarray(B, np.int8)
    out = np.array(Cbuf, dtype=np.int32, copy=True)
    _lib.ora_igemm_npu(m, n, k, alpha, beta, _p(A), lda, _p(B), ldb, _p(out), ldc)
    return out


def gemm_f64(ta, tb, m, n, k, alpha, A, lda, B, ldb, beta=0.0, Cin=None, ldc=None, sA=0, sB=0, sC=0, batch=1,
             bias=None, sBias=0, scale_mode=0, sa=None, sb=None, ssa=0, ssb=0, j0=0, j1=None, nthreads=None,
             out=None) -> np.ndarray:
    """fp64 D = alpha*s*op(A)op(B) + beta*Cin + bias over columns [j0, j1); A/B are float arrays
    holding the exact decoded input values. Returns the column-major fp64 buffer."""
    ldc = m if ldc is None else ldc
    j1 = n if j1 is None else j1
    A = np.ascontiguousarray(A, np.float32)
    B = np.ascontiguousarray(B, np.float32)
    size = (batch - 1) * sC + ldc * n if batch > 1 else ldc * n
    if out is None:
        out = np.zeros(size, dtype=np.float64)
    cin = None if Cin is None else np.ascontiguousarray(Cin, np.float64)
    bias = None if bias is None else np.ascontiguousarray(bias, np.float32)
    sa = None if sa is None else np.ascontiguousarray(sa, np.float32)
    sb = None if sb is None else np.ascontiguousarray(sb, np.float32)
    _lib.ora_gemm_f64(int(ta), int(tb), m, n, k, alpha, _p(A), lda, sA, _p(B), ldb, sB, beta, _p(cin), _p(out), ldc,
                      sC, batch, _p(bias), sBias, scale_mode, _p(sa), _p(sb), ssa, ssb, j0, j1,
                      nthreads or nthreads_default())
    return out


# ------------------------------------------------------------ norms / attention

def rmsnorm(x, gamma, eps, nthreads=None):
    x = np.ascontiguousarray(x, np.float32)
    gamma = np.ascontiguousarray(gamma, np.float32)
    rows, hidden = x.shape
    y = np.empty((rows, hidden), np.float64)
    rstd = np.empty(rows, np.float64)
    _lib.ora_rmsnorm(rows, hidden, _p(x), hidden, _p(gamma), eps, _p(y), _p(rstd), nthreads or nthreads_default())
    return y, rstd


def norm_bwd(ln, x, dy, gamma, eps):
    """fp64 RMSNorm (ln=False) / LayerNorm (ln=True) backward: (dx, dgamma, dbeta or None)."""
    x = np.ascontiguousarray(x, np.float32)
    dy = np.ascontiguousarray(dy, np.float32)
    gamma = np.ascontiguousarray(gamma, np.float32)
    rows, hidden = x.shape
    dx = np.empty((rows, hidden), np.float64)
    dg = np.empty(hidden, np.float64)
    db = np.empty(hidden, np.float64) if ln else None
    _lib.ora_norm_bwd(1 if ln else 0, rows, hidden, _p(x), _p(dy), _p(gamma), eps, _p(dx), _p(dg), _p(db))
    return dx, dg, db


def layernorm(x, gamma, beta, eps, nthreads=None):
    x = np.ascontiguousarray(x, np.float32)
    gamma = np.ascontiguousarray(gamma, np.float32)
    beta = None if beta is None else np.ascontiguousarray(beta, np.float32)
    rows, hidden = x.shape
    y = np.empty((rows, hidden), np.float64)
    mean = np.empty(rows, np.float64)
    rstd = np.empty(rows, np.float64)
    _lib.ora_layernorm(rows, hidden, _p(x), hidden, _p(gamma), _p(beta), eps, _p(y), _p(mean), _p(rstd),
                       nthreads or nthreads_default())
    return y, mean, rstd


def attention(q, k, v, scale, causal, pairs=None, q0=0, q1=None, nthreads=None):
    """q: [BH, Sq, D], k/v: [BH, Sk, D] float arrays. Returns (o [P, nq, D], lse [P, nq])."""
    q = np.ascontiguousarray(q, np.float32)
    k = np.ascontiguousarray(k, np.float32)
    v = np.ascontiguousarray(v, np.float32)
    BH, Sq, D = q.shape
    Sk = k.shape[1]
    pairs = np.arange(BH, dtype=np.int32) if pairs is None else np.ascontiguousarray(pairs, np.int32)
    q1 = Sq if q1 is None else q1
    nq = q1 - q0
    o = np.empty((len(pairs), nq, D), np.float64)
    lse = np.empty((len(pairs), nq), np.float64)
    _lib.ora_attention(BH, Sq, Sk, D, _p(q), _p(k), _p(v), scale, int(causal), _p(pairs), len(pairs), q0, q1, _p(o),
                       _p(lse), nthreads or nthreads_default())
    return o, lse


def attention_bwd(q, k, v, dout, scale, causal, nthreads=None):
    """q, dout: [BH, Sq, D]; k, v: [BH, Sk, D] float arrays. Returns fp64 (dq, dk, dv)."""
    q, k, v, dout = (np.ascontiguousarray(t, np.float32) for t in (q, k, v, dout))
    BH, Sq, D = q.shape
    Sk = k.shape[1]
    dq = np.empty((BH, Sq, D), np.float64)
    dk = np.empty((BH, Sk, D), np.float64)
    dv = np.empty((BH, Sk, D), np.float64)
    _lib.ora_attention_bwd(BH, Sq, Sk, D, _p(q), _p(k), _p(v), _p(dout), scale, int(causal), _p(dq), _p(dk), _p(dv),
                           nthreads or nthreads_default())
    return dq, dk, dv


def conv2d(x, w, pad=(0, 0), stride=(1, 1), dilation=(1, 1)):
    """fp64 conv2d: x [n, h, w, c] NHWC, w [k, r, s, c] KRSC -> y [n, p, q, k]."""
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    n, h, wd, c = x.shape
    k, r, s, _ = w.shape
    P = (h + 2 * pad[0] - dilation[0] * (r - 1) - 1) // stride[0] + 1
    Q = (wd + 2 * pad[1] - dilation[1] * (s - 1) - 1) // stride[1] + 1
    y = np.empty((n, P, Q, k), np.float64)
    _lib.ora_conv2d(n, h, wd, c, k, r, s, pad[0], pad[1], stride[0], stride[1], dilation[0], dilation[1], P, Q, _p(x),
                    _p(w), _p(y))
    return y


def pool2d(x, window, pad=(0, 0), stride=None, mode=0):
    """fp64 NHWC pooling: mode 0 max (0 for an all-padding window), 1 average over r*s,
    2 average over the in-image taps."""
    x = np.asarray(x, np.float64)
    n, h, wd, c = x.shape
    r, s = window
    st = stride or window
    P = (h + 2 * pad[0] - r) // st[0] + 1
    Q = (wd + 2 * pad[1] - s) // st[1] + 1
    y = np.zeros((n, P, Q, c))
    for p in range(P):
        for q in range(Q):
            h0, w0 = p * st[0] - pad[0], q * st[1] - pad[1]
            win = x[:, max(h0, 0):min(h0 + r, h), max(w0, 0):min(w0 + s, wd), :]
            cnt = win.shape[1] * win.shape[2]
            if cnt == 0:
                continue
            if mode == 0:
                y[:, p, q, :] = win.max(axis=(1, 2))
            elif mode == 1:
                y[:, p, q, :] = win.sum(axis=(1, 2)) / (r * s)
            else:
                y[:, p, q, :] = win.sum(axis=(1, 2)) / cnt
    return y


# ------------------------------------------------------------ level 1 / 2

def saxpy(n, alpha, x, incx, y, incy):
    """tests/libs/test_grxblas_l12.cpp:79-92; returns the new y buffer."""
    x = np.ascontiguousarray(x, np.float32)
    out = np.array(y, dtype=np.float32, copy=True)
    _lib.ora_saxpy(n, alpha, _p(x), incx, _p(out), incy)
    return out


def sscal(n, alpha, x, incx):
    out = np.array(x, dtype=np.float32, copy=True)
    _lib.ora_sscal(n, alpha, _p(out), incx)
    return out


def sgemv(trans, m, n, alpha, A, lda, x, incx, beta, y, incy):
    A = np.ascontiguousarray(A, np.float32)
    x = np.ascontiguousarray(x, np.float32)
    out = np.array(y, dtype=np.float32, copy=True)
    _lib.ora_sgemv(int(trans), m, n, alpha, _p(A), lda, _p(x), incx, beta, _p(out), incy)
    return out


def softmax(x):
    """Row softmax of a [rows, cols] float array in fp64 (definition)."""
    x = np.ascontiguousarray(x, np.float32)
    rows, cols = x.shape
    y = np.empty((rows, cols), np.float64)
    _lib.ora_softmax(rows, cols, _p(x), cols, _p(y))
    return y


def softmax_bwd(y, dy):
    """fp64 softmax backward from the forward output: dx = y (dy - sum_c dy y)."""
    y = np.asarray(y, np.float64)
    dy = np.asarray(dy, np.float64)
    return y * (dy - (dy * y).sum(axis=-1, keepdims=True))


def gelu_bwd(x, dy, mode=0):
    """fp64 dy * GELU'(x): mode 0 erf form Phi(x) + x phi(x), 1 the tanh approximation's derivative."""
    from math import erf, pi, sqrt

    x = np.asarray(x, np.float64)
    dy = np.asarray(dy, np.float64)
    if mode == 0:
        cdf = 0.5 * (1.0 + np.vectorize(erf)(x / sqrt(2.0)))
        pdf = np.exp(-0.5 * x * x) / sqrt(2.0 * pi)
        return dy * (cdf + x * pdf)
    k0 = sqrt(2.0 / pi)
    t = np.tanh(k0 * (x + 0.044715 * x ** 3))
    return dy * (0.5 * (1.0 + t) + 0.5 * x * (1.0 - t * t) * k0 * (1.0 + 3.0 * 0.044715 * x * x))


def gelu(x, mode=0):
    """GELU in fp64: mode 0 erf form, 1 tanh approximation."""
    x = np.ascontiguousarray(x, np.float32)
    y = np.empty(x.shape, np.float64)
    _lib.ora_gelu(x.size, _p(x), _p(y), mode)
    return y
