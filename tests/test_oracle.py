"""Pins the oracle before anything is checked against it (CPU only).

* fp32 sgemm: the oracle's restatements against the outputs of the reference's
  own sgemm kernel source compiled for this host (tests/golden/ref_sgemm.npz,
  made by tests/golden/make_golden.py from oracle/_ref): the kernel restatement
  must agree bit for bit, the fp64 gate reference within the reference's own
  bound 1e-5*(k+1) (tests/libs/test_grxblas.cpp:234).
* int8: the reference's known-answer GEMMs (src/backends/npu_c930/
  test_npu_c930.cc:183-230), and the NPU test's int64-accumulate reference
  (tests/libs/test_grxblas_npu.cpp:50-66) against the column-major int32 gate.
* fp16 GemmEx: on the reference's exact inputs (tests/libs/test_grxblas_ex.cpp:
  1-14) the fp32-sequential gate equals the fp64 product exactly.
* conversions: bf16 / fp16 / e4m3 rounding against PyTorch's casts, bit for bit.
* norms / attention: fp64 definitions checked against independent numpy code.
"""
from __future__ import annotations

import os
import subprocess
from pathlib import Path

import numpy as np
import pytest
import torch

import oracle
from gates import SGEMM_BATCHED_CASES, SGEMM_CASES, HalfSampler, gemmex_cases, int8_patterns, lcg_fill

ROOT = Path(__file__).resolve().parent.parent
GOLDEN = np.load(ROOT / "tests/golden/ref_sgemm.npz")


@pytest.mark.parametrize("case", SGEMM_CASES, ids=[c[-1] for c in SGEMM_CASES])
def test_sgemm_oracle_matches_reference_kernel(case):
    ta, tb, m, n, k, alpha, beta, pad, label = case
    lda, ldb, ldc = max(1, (k if ta else m) + pad), max(1, (n if tb else k) + pad), max(1, m + pad)
    A = lcg_fill(lda * (m if ta else k), 1)
    B = lcg_fill(ldb * (k if tb else n), 7)
    C = lcg_fill(ldc * n, 13)
    ref = GOLDEN["single/" + label]
    kern = oracle.sgemm_kernel(ta, tb, m, n, k, alpha, A, lda, 0, B, ldb, 0, beta, C, ldc, 0, 1)
    assert np.array_equal(kern, ref)
    gate = oracle.sgemm_ref(ta, tb, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc)
    assert np.all(np.abs(gate - ref) <= 1e-5 * (k + 1))


@pytest.mark.parametrize("case", SGEMM_BATCHED_CASES, ids=[c[-1] for c in SGEMM_BATCHED_CASES])
def test_sgemm_batched_oracle_matches_reference_kernel(case):
    ta, tb, m, n, k, alpha, beta, batch, gap, bcast, label = case
    lda, ldb, ldc = max(1, k if ta else m), max(1, n if tb else k), max(1, m)
    ae, be, ce = lda * (m if ta else k), ldb * (k if tb else n), ldc * n
    sa, sb, sc = ae + gap, 0 if bcast else be + gap, ce + gap
    A = lcg_fill(sa * (batch - 1) + ae + gap, 3)
    B = lcg_fill(be + gap if bcast else sb * (batch - 1) + be + gap, 11)
    C = lcg_fill(sc * (batch - 1) + ce + gap, 17)
    got = oracle.sgemm_kernel(ta, tb, m, n, k, alpha, A, lda, sa, B, ldb, sb, beta, C, ldc, sc, batch)
    assert np.array_equal(got, GOLDEN["batched/" + label])


def test_reference_kernel_live_when_available():
    """Re-runs the reference-built kernel (oracle/_ref) when it is present, so the
    committed fixture cannot drift from the code it was made from."""
    lib = ROOT / "oracle/_ref/libref_sgemm.so"
    if not lib.exists():
        pytest.skip("oracle/_ref not built on this machine")
    import ctypes as C

    f = C.CDLL(str(lib)).ref_sgemm_run
    vp, i, ll, fl = C.c_void_p, C.c_int, C.c_longlong, C.c_float
    f.argtypes = [i, i, i, i, i, fl, vp, i, ll, vp, i, ll, fl, vp, i, ll, i]
    rng = np.random.default_rng(0)
    for ta, tb in [(0, 0), (1, 0), (0, 1), (1, 1)]:
        m, n, k = 33, 21, 47
        lda, ldb, ldc = (k if ta else m) + 2, (n if tb else k) + 1, m + 3
        A = rng.standard_normal(lda * (m if ta else k)).astype(np.float32)
        B = rng.standard_normal(ldb * (k if tb else n)).astype(np.float32)
        Cb = rng.standard_normal(ldc * n).astype(np.float32)
        want = oracle.sgemm_kernel(ta, tb, m, n, k, 1.5, A, lda, 0, B, ldb, 0, -0.5, Cb, ldc, 0, 1)
        out = Cb.copy()
        f(ta, tb, m, n, k, 1.5, A.ctypes.data, lda, 0, B.ctypes.data, ldb, 0, -0.5, out.ctypes.data, ldc, 0, 1)
        assert np.array_equal(out, want)


def test_reference_npu_unit_test_passes_when_available():
    exe = ROOT / "oracle/_ref/test_npu_c930"
    if not exe.exists():
        pytest.skip("oracle/_ref not built on this machine")
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0 and "ALL PASSED" in r.stdout


def test_int8_known_answers():
    # src/backends/npu_c930/test_npu_c930.cc:183-230 (row-major 2x2x2)
    A = np.array([1, 2, 3, 4], np.int8)
    B = np.array([5, 6, 7, 8], np.int8)
    got = oracle.igemm_npu(2, 2, 2, 1, 0, A, 2, B, 2, np.zeros(4, np.int32), 2)
    assert got.tolist() == [19, 22, 43, 50]
    A = np.array([-1, 2, 3, -4], np.int8)
    B = np.array([5, -6, 7, 8], np.int8)
    got = oracle.igemm_npu(2, 2, 2, 1, 0, A, 2, B, 2, np.zeros(4, np.int32), 2)
    assert got.tolist() == [9, 22, -13, -50]
    # the column-major int32 gate agrees: row-major C = A B is column-major C^T = B^T A^T
    A = np.array([1, 2, 3, 4], np.int8)
    B = np.array([5, 6, 7, 8], np.int8)
    got = oracle.igemm(0, 0, 2, 2, 2, 1, B, 2, A, 2, 0, np.zeros(4, np.int32), 2)
    assert got.tolist() == [19, 22, 43, 50]


@pytest.mark.parametrize("ta,tb", [(0, 0), (1, 0), (0, 1), (1, 1)])
def test_int8_gate_vs_int64_reference(ta, tb):
    m, n, k, pad = 17, 9, 29, 3
    a_rows, a_cols = (k, m) if ta else (m, k)
    b_rows, b_cols = (n, k) if tb else (k, n)
    lda, ldb, ldc = a_rows + pad, b_rows + pad, m + pad
    A, B, C = int8_patterns(lda * a_cols, ldb * b_cols, ldc * n)
    got = oracle.igemm(ta, tb, m, n, k, 2, A, lda, B, ldb, -1, C, ldc)
    # independent int64 computation
    Am = np.array([[A[l + i * lda] if ta else A[i + l * lda] for l in range(k)] for i in range(m)], np.int64)
    Bm = np.array([[B[j + l * ldb] if tb else B[l + j * ldb] for j in range(n)] for l in range(k)], np.int64)
    want = C.astype(np.int64).copy()
    prod = Am @ Bm
    for j in range(n):
        for i in range(m):
            want[i + j * ldc] = 2 * prod[i, j] - C[i + j * ldc]
    assert np.array_equal(got, want.astype(np.int32))


def test_int32_wraparound_is_twos_complement():
    A = np.full(4, 127, np.int8)
    B = np.full(4, 127, np.int8)
    C = np.array([2 ** 31 - 1], np.int32)
    got = oracle.igemm(0, 0, 1, 1, 4, 1, A, 1, B, 4, 1, C, 1)
    assert got[0] == np.int32(np.int64(2 ** 31 - 1 + 4 * 127 * 127) - 2 ** 32)


@pytest.mark.parametrize("case", gemmex_cases(128, 256, 64)[:9], ids=[c[-1] for c in gemmex_cases(128, 256, 64)[:9]])
def test_fp16_gate_is_exact(case):
    ta, tb, m, n, k, alpha, beta, pad, _ = case
    kk = k if k else 1
    a_rows, a_cols = (kk, m) if ta else (m, kk)
    b_rows, b_cols = (n, kk) if tb else (kk, n)
    lda, ldb, ldc = a_rows + pad, b_rows + pad, m + pad
    s = HalfSampler(99)
    A, B = s.take(lda * a_cols), s.take(ldb * b_cols)
    C = s.take(ldc * n) * np.float32(2)
    for kind in ("f16", "bf16"):
        assert np.array_equal(oracle.round_to(kind, A), A)
    f32 = oracle.gemm_f32seq(ta, tb, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc)
    f64 = oracle.gemm_f64(ta, tb, m, n, k, alpha, A, lda, B, ldb, beta=beta, Cin=C.astype(np.float64), ldc=ldc)
    inside = np.zeros(C.size, bool)
    for j in range(n):
        inside[j * ldc:j * ldc + m] = True
    assert np.array_equal(f32[inside], f64[inside].astype(np.float32))


def test_conversions_match_torch():
    torch = pytest.importorskip("torch")
    x = np.random.default_rng(0).standard_normal(200000).astype(np.float32) * np.float32(50)
    x = np.concatenate([x, np.array([0.0, -0.0, 1e-8, -1e-8, 65504, 65520, 1e30], np.float32)])
    assert np.array_equal(oracle.round_to("bf16", x), torch.from_numpy(x).bfloat16().float().numpy())
    assert np.array_equal(oracle.round_to("f16", x), torch.from_numpy(x).half().float().numpy())
    xs = np.clip(x, -448, 448)
    assert np.array_equal(oracle.round_to("e4m3", xs), torch.from_numpy(xs).to(torch.float8_e4m3fn).float().numpy())
    sub = (np.random.default_rng(1).standard_normal(50000) * 1e-2).astype(np.float32)
    assert np.array_equal(oracle.round_to("e4m3", sub), torch.from_numpy(sub).to(torch.float8_e4m3fn).float().numpy())
    assert oracle.round_to("e4m3", np.array([1000.0, -1000.0], np.float32)).tolist() == [448.0, -448.0]


def test_fp64_gemm_epilogue_and_threads():
    rng = np.random.default_rng(3)
    m, n, k = 37, 23, 41
    A = rng.standard_normal(m * k).astype(np.float32)
    B = rng.standard_normal(k * n).astype(np.float32)
    bias = rng.standard_normal(n).astype(np.float32)
    sa = rng.random(m).astype(np.float32)
    sb = rng.random(n).astype(np.float32)
    Cin = rng.standard_normal(m * n)
    got1 = oracle.gemm_f64(0, 0, m, n, k, 1.5, A, m, B, k, beta=0.5, Cin=Cin, bias=bias, scale_mode=2, sa=sa, sb=sb,
                           nthreads=1)
    got4 = oracle.gemm_f64(0, 0, m, n, k, 1.5, A, m, B, k, beta=0.5, Cin=Cin, bias=bias, scale_mode=2, sa=sa, sb=sb,
                           nthreads=4)
    Am = A.reshape(k, m).T.astype(np.float64)
    Bm = B.reshape(n, k).T.astype(np.float64)
    want = 1.5 * sa[:, None].astype(np.float64) * sb[None, :] * (Am @ Bm) + 0.5 * Cin.reshape(n, m).T + bias[None, :]
    assert np.array_equal(got1, got4)
    assert np.allclose(got1.reshape(n, m).T, want, rtol=1e-12, atol=1e-12)


def test_norms_match_numpy():
    rng = np.random.default_rng(4)
    x = rng.standard_normal((9, 300)).astype(np.float32)
    g = rng.standard_normal(300).astype(np.float32)
    b = rng.standard_normal(300).astype(np.float32)
    y, r = oracle.rmsnorm(x, g, 1e-5)
    xd = x.astype(np.float64)
    assert np.allclose(y, xd / np.sqrt((xd ** 2).mean(1, keepdims=True) + 1e-5) * g, rtol=1e-12)
    y, mu, rs = oracle.layernorm(x, g, b, 1e-5)
    want = (xd - xd.mean(1, keepdims=True)) / np.sqrt(xd.var(1, keepdims=True) + 1e-5) * g + b
    assert np.allclose(y, want, rtol=1e-11, atol=1e-12)


@pytest.mark.parametrize("causal", [False, True])
def test_attention_matches_numpy(causal):
    rng = np.random.default_rng(5)
    BH, S, D = 3, 50, 16
    q, k, v = (rng.standard_normal((BH, S, D)).astype(np.float32) for _ in range(3))
    o, lse = oracle.attention(q, k, v, 0.25, causal)
    s = np.einsum("bqd,bkd->bqk", q.astype(np.float64), k.astype(np.float64)) * 0.25
    if causal:
        s = np.where(np.tril(np.ones((S, S), bool))[None], s, -np.inf)
    mx = s.max(-1, keepdims=True)
    p = np.exp(s - mx)
    l = p.sum(-1, keepdims=True)
    assert np.allclose(o, (p / l) @ v.astype(np.float64), rtol=1e-10, atol=1e-12)
    assert np.allclose(lse, (mx + np.log(l))[..., 0], rtol=1e-12)
    o2, l2 = oracle.attention(q, k, v, 0.25, causal, pairs=[2], q0=10, q1=20)
    assert np.allclose(o2[0], o[2, 10:20]) and np.allclose(l2[0], lse[2, 10:20])


@pytest.mark.parametrize("ln", [False, True])
def test_norm_backward_oracle_matches_autograd(ln):
    """The fp64 norm-backward restatement against torch autograd in fp64
    (an independent derivation of the same derivative)."""
    rng = np.random.default_rng(11)
    x = rng.standard_normal((5, 48)).astype(np.float32)
    dy = rng.standard_normal((5, 48)).astype(np.float32)
    g = rng.standard_normal(48).astype(np.float32)
    dx, dg, db = oracle.norm_bwd(ln, x, dy, g, 1e-5)
    X = torch.tensor(x, dtype=torch.float64, requires_grad=True)
    G = torch.tensor(g, dtype=torch.float64, requires_grad=True)
    Bt = torch.zeros(48, dtype=torch.float64, requires_grad=True)
    if ln:
        y = torch.nn.functional.layer_norm(X, (48,), G, Bt, 1e-5)
    else:
        y = X * torch.rsqrt((X * X).mean(1, keepdim=True) + 1e-5) * G
    y.backward(torch.tensor(dy, dtype=torch.float64))
    assert np.allclose(dx, X.grad.numpy(), rtol=1e-12, atol=1e-12)
    assert np.allclose(dg, G.grad.numpy(), rtol=1e-12, atol=1e-12)
    if ln:
        assert np.allclose(db, Bt.grad.numpy(), rtol=1e-12, atol=1e-12)


@pytest.mark.parametrize("causal,sq,sk", [(True, 7, 7), (False, 5, 9)])
def test_attention_backward_oracle_matches_autograd(causal, sq, sk):
    """The fp64 attention-backward restatement against torch autograd in fp64."""
    rng = np.random.default_rng(5)
    q = rng.standard_normal((2, sq, 16)).astype(np.float32)
    k = rng.standard_normal((2, sk, 16)).astype(np.float32)
    v = rng.standard_normal((2, sk, 16)).astype(np.float32)
    do = rng.standard_normal((2, sq, 16)).astype(np.float32)
    dq, dk, dv = oracle.attention_bwd(q, k, v, do, 0.3, causal)
    Q, K, V = (torch.tensor(t, dtype=torch.float64, requires_grad=True) for t in (q, k, v))
    s = Q @ K.transpose(1, 2) * 0.3
    if causal:
        s = s.masked_fill(torch.ones(sq, sk, dtype=torch.bool).triu(1), float("-inf"))
    (torch.softmax(s, -1) @ V).backward(torch.tensor(do, dtype=torch.float64))
    for got, ref in ((dq, Q.grad), (dk, K.grad), (dv, V.grad)):
        assert np.allclose(got, ref.numpy(), rtol=1e-10, atol=1e-12)


@pytest.mark.parametrize("pad,stride,dil", [((0, 0), (1, 1), (1, 1)), ((1, 2), (2, 1), (1, 2))])
def test_conv2d_oracle_matches_torch(pad, stride, dil):
    """The fp64 conv restatement (NHWC / KRSC) against torch's conv2d in fp64 (NCHW)."""
    rng = np.random.default_rng(3)
    x = rng.standard_normal((2, 9, 11, 5)).astype(np.float32)
    w = rng.standard_normal((4, 3, 2, 5)).astype(np.float32)
    y = oracle.conv2d(x, w, pad, stride, dil)
    ref = torch.nn.functional.conv2d(torch.tensor(x, dtype=torch.float64).permute(0, 3, 1, 2),
                                     torch.tensor(w, dtype=torch.float64).permute(0, 3, 1, 2),
                                     stride=stride, padding=pad, dilation=dil).permute(0, 2, 3, 1).numpy()
    assert y.shape == ref.shape and np.allclose(y, ref, rtol=1e-12, atol=1e-12)


def test_pool2d_oracle_matches_torch():
    rng = np.random.default_rng(4)
    x = rng.standard_normal((2, 9, 10, 3))
    t = torch.tensor(x).permute(0, 3, 1, 2)
    mx = torch.nn.functional.max_pool2d(t, 3, 2, 1).permute(0, 2, 3, 1).numpy()
    av = torch.nn.functional.avg_pool2d(t, 3, 2, 1, count_include_pad=True).permute(0, 2, 3, 1).numpy()
    ex = torch.nn.functional.avg_pool2d(t, 3, 2, 1, count_include_pad=False).permute(0, 2, 3, 1).numpy()
    assert np.allclose(oracle.pool2d(x, (3, 3), (1, 1), (2, 2), 0), mx)
    assert np.allclose(oracle.pool2d(x, (3, 3), (1, 1), (2, 2), 1), av)
    assert np.allclose(oracle.pool2d(x, (3, 3), (1, 1), (2, 2), 2), ex)


@pytest.mark.parametrize("mode", [0, 1])
def test_softmax_gelu_backward_oracle_match_autograd(mode):
    """The fp64 softmax / GELU backward restatements against torch autograd in fp64."""
    rng = np.random.default_rng(21)
    x = rng.standard_normal((4, 37)) * 3
    dy = rng.standard_normal((4, 37))
    X = torch.tensor(x, requires_grad=True)
    torch.softmax(X, -1).backward(torch.tensor(dy))
    y = torch.softmax(torch.tensor(x), -1).numpy()
    assert np.allclose(oracle.softmax_bwd(y, dy), X.grad.numpy(), rtol=1e-12, atol=1e-14)
    X = torch.tensor(x, requires_grad=True)
    torch.nn.functional.gelu(X, approximate="none" if mode == 0 else "tanh").backward(torch.tensor(dy))
    assert np.allclose(oracle.gelu_bwd(x, dy, mode), X.grad.numpy(), rtol=1e-12, atol=1e-14)
