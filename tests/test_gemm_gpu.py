"""GPU parity of grxBLAS GEMM against the oracle, through the C-ABI.

Mirrors the reference's gates (tests/libs/test_grxblas.cpp, test_grxblas_ex.cpp):
whole-buffer comparisons including ld padding (a stray write is a failure),
ragged shapes, every transpose, alpha/beta, k = 0, strided batches with slack
and broadcast. fp32 sgemm: the reference's per-element bound 1e-5*(k+1)
(test_grxblas.cpp:234). fp16/bf16 GemmEx on exact inputs and int8 -> int32:
bit-exact (test_grxblas_ex.cpp:131, :267-281). bf16 / fp8 / scaled int8:
|got - ref| <= 1e-2 + 2e-2*|ref| against the fp64 oracle (BASELINE tolerance).
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from gates import (SGEMM_BATCHED_CASES, SGEMM_CASES, HalfSampler, gemmex_cases, int8_cases, int8_patterns,
                   lcg_fill)
from grxcp_b200 import _native as N

pytestmark = pytest.mark.gpu

TOL_ABS, TOL_REL = 1e-2, 2e-2


def dev_f32(a):
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda()


def dev_bits(bits):
    b = np.ascontiguousarray(bits)
    if b.dtype == np.uint16:
        return torch.from_numpy(b.view(np.int16)).cuda()
    if b.dtype == np.uint8:
        return torch.from_numpy(b.view(np.int8)).cuda()
    return torch.from_numpy(b).cuda()


def nonempty(t, dtype=torch.float32):
    return t if t.numel() else torch.zeros(1, dtype=dtype, device="cuda")


def close(got, ref):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    bad = np.abs(got - ref) > TOL_ABS + TOL_REL * np.abs(ref)
    return not bad.any(), int(bad.sum())


# ------------------------------------------------------------------ sgemm

@pytest.mark.parametrize("case", SGEMM_CASES, ids=[c[-1] for c in SGEMM_CASES])
def test_sgemm_reference_cases(blas, case):
    ta, tb, m, n, k, alpha, beta, pad, _ = case
    lda = max(1, (k if ta else m) + pad)
    ldb = max(1, (n if tb else k) + pad)
    ldc = max(1, m + pad)
    A = lcg_fill(lda * (m if ta else k), 1)
    B = lcg_fill(ldb * (k if tb else n), 7)
    C = lcg_fill(ldc * n, 13)
    want = oracle.sgemm_ref(ta, tb, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc)
    dA, dB, dC = nonempty(dev_f32(A)), nonempty(dev_f32(B)), dev_f32(C)
    assert blas.sgemm(ta, tb, m, n, k, alpha, dA, lda, dB, ldb, beta, dC, ldc) == N.SUCCESS
    torch.cuda.synchronize()
    got = dC.cpu().numpy()
    idx = np.arange(C.size)
    inside = ((idx % ldc) < m) & ((idx // ldc) < n)
    assert np.array_equal(got[~inside], want[~inside]), "stray write outside the m x n window"
    assert np.all(np.abs(got[inside] - want[inside]) <= 1e-5 * (k + 1))


@pytest.mark.parametrize("case", SGEMM_BATCHED_CASES, ids=[c[-1] for c in SGEMM_BATCHED_CASES])
def test_sgemm_strided_batched(blas, case):
    ta, tb, m, n, k, alpha, beta, batch, gap, bcast, _ = case
    lda, ldb, ldc = max(1, k if ta else m), max(1, n if tb else k), max(1, m)
    ae, be, ce = lda * (m if ta else k), ldb * (k if tb else n), ldc * n
    sa, sb, sc = ae + gap, 0 if bcast else be + gap, ce + gap
    A = lcg_fill(sa * (batch - 1) + ae + gap, 3)
    B = lcg_fill(be + gap if bcast else sb * (batch - 1) + be + gap, 11)
    C = lcg_fill(sc * (batch - 1) + ce + gap, 17)
    want = oracle.sgemm_kernel(ta, tb, m, n, k, alpha, A, lda, sa, B, ldb, sb, beta, C, ldc, sc, batch)
    ref64 = C.copy()
    for bi in range(batch):
        ref64[sc * bi:] = oracle.sgemm_ref(ta, tb, m, n, k, alpha, A[sa * bi:], lda, B[sb * bi:], ldb, beta,
                                           ref64[sc * bi:], ldc)
    dA, dB, dC = dev_f32(A), dev_f32(B), dev_f32(C)
    assert blas.sgemm_strided_batched(ta, tb, m, n, k, alpha, dA, lda, sa, dB, ldb, sb, beta, dC, ldc, sc,
                                      batch) == N.SUCCESS
    torch.cuda.synchronize()
    got = dC.cpu().numpy()
    assert np.all(np.abs(got - ref64) <= 1e-5 * (k + 1))
    assert np.all(np.abs(got - want) <= 1e-5 * (k + 1))


def test_sgemm_512_config(blas):
    """row-major 512^3 via the swapped column-major call, U[-1, 1]."""
    rng = np.random.default_rng(1)
    M = N_ = K = 512
    A = rng.uniform(-1, 1, (M, K)).astype(np.float32)  # row-major
    B = rng.uniform(-1, 1, (K, N_)).astype(np.float32)
    # row-major C = A B  <=>  column-major C^T = B^T A^T: call with (B, A), m = N, n = M
    want = oracle.sgemm_ref(0, 0, N_, M, K, 1.0, B.ravel(), N_, A.ravel(), K, 0.0, np.zeros(M * N_, np.float32), N_)
    dA, dB = dev_f32(A.ravel()), dev_f32(B.ravel())
    dC = torch.full((M * N_,), float("nan"), device="cuda")
    assert blas.sgemm(0, 0, N_, M, K, 1.0, dB, N_, dA, K, 0.0, dC, N_) == N.SUCCESS
    torch.cuda.synchronize()
    got = dC.cpu().numpy()
    rel = np.abs(got - want).max() / np.abs(want).max()
    assert rel <= 1e-5
    assert np.all(np.abs(got - want) <= 1e-5 * (K + 1))


# ------------------------------------------------------------------ GemmEx exact

def _ex_case(blas, ta, tb, m, n, k, alpha, beta, pad, kind, grx_type):
    kk = k if k else 1
    a_rows, a_cols = (kk, m) if ta else (m, kk)
    b_rows, b_cols = (n, kk) if tb else (kk, n)
    lda, ldb, ldc = a_rows + pad, b_rows + pad, m + pad
    smp = HalfSampler(99)
    A = smp.take(lda * a_cols)
    B = smp.take(ldb * b_cols)
    C = smp.take(ldc * n) * np.float32(2)
    assert np.array_equal(oracle.round_to(kind, A), A) and np.array_equal(oracle.round_to(kind, B), B)
    want = oracle.gemm_f32seq(ta, tb, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc)
    dA, dB, dC = dev_bits(oracle.encode(kind, A)), dev_bits(oracle.encode(kind, B)), dev_f32(C)
    st = blas.gemm_ex(ta, tb, m, n, k, alpha, dA, grx_type, lda, dB, grx_type, ldb, beta, dC, N.GRX_R_32F, ldc)
    assert st == N.SUCCESS, N.STATUS[st]
    torch.cuda.synchronize()
    assert blas.execution_status() == N.SUCCESS
    got = dC.cpu().numpy()
    diff = np.nonzero(got != want)[0]
    assert diff.size == 0, f"{diff.size} mismatches, first at {diff[:3]}: got {got[diff[:3]]} want {want[diff[:3]]}"


TILE = (128, 256, 64)


@pytest.mark.parametrize("case", gemmex_cases(*TILE), ids=[c[-1] for c in gemmex_cases(*TILE)])
def test_gemmex_fp16_exact(blas, case):
    ta, tb, m, n, k, alpha, beta, pad, _ = case
    _ex_case(blas, ta, tb, m, n, k, alpha, beta, pad, "f16", N.GRX_R_16F)


@pytest.mark.parametrize("case", gemmex_cases(*TILE), ids=[c[-1] for c in gemmex_cases(*TILE)])
def test_gemmex_bf16_exact(blas, case):
    ta, tb, m, n, k, alpha, beta, pad, _ = case
    _ex_case(blas, ta, tb, m, n, k, alpha, beta, pad, "bf16", N.GRX_R_16BF)


def test_tensor_tile_and_types(blas):
    s, tile = blas.tensor_tile()
    assert s == N.SUCCESS and tile == TILE
    s, mask = blas.tensor_types()
    assert s == N.SUCCESS and mask & 0x01 and mask & 0x10 and mask & 0x40 and mask & 0x04


@pytest.mark.parametrize("case", int8_cases(128, 256), ids=[c[-1] for c in int8_cases(128, 256)])
def test_gemmex_int8_exact(blas, case):
    ta, tb, m, n, k, alpha, beta, pad, _ = case
    kk = k if k else 1
    a_rows, a_cols = (kk, m) if ta else (m, kk)
    b_rows, b_cols = (n, kk) if tb else (kk, n)
    lda, ldb, ldc = a_rows + pad, b_rows + pad, m + pad
    A, B, C = int8_patterns(lda * a_cols, ldb * b_cols, ldc * n)
    want = oracle.igemm(ta, tb, m, n, k, int(alpha), A, lda, B, ldb, int(beta), C, ldc)
    dA, dB, dC = dev_bits(A), dev_bits(B), torch.from_numpy(C.copy()).cuda()
    st = blas.gemm_ex(ta, tb, m, n, k, alpha, dA, N.GRX_R_8I, lda, dB, N.GRX_R_8I, ldb, beta, dC, N.GRX_R_32I, ldc)
    assert st == N.SUCCESS, N.STATUS[st]
    torch.cuda.synchronize()
    assert np.array_equal(dC.cpu().numpy(), want)


def test_gemmex_int8_512_random(blas):
    """BASELINE config 1, int8 variant: uniform ints in [-128, 127], 512^3, bit-exact int32."""
    rng = np.random.default_rng(5)
    m = n = k = 512
    A = rng.integers(-128, 128, m * k).astype(np.int8)
    B = rng.integers(-128, 128, k * n).astype(np.int8)
    C = np.zeros(m * n, np.int32)
    for ta, tb in [(0, 0), (1, 0), (0, 1), (1, 1)]:
        want = oracle.igemm(ta, tb, m, n, k, 1, A, 512, B, 512, 0, C, m)
        dC = torch.full((m * n,), -1, dtype=torch.int32, device="cuda")
        st = blas.gemm_ex(ta, tb, m, n, k, 1.0, dev_bits(A), N.GRX_R_8I, 512, dev_bits(B), N.GRX_R_8I, 512, 0.0, dC,
                          N.GRX_R_32I, m)
        assert st == N.SUCCESS
        torch.cuda.synchronize()
        assert np.array_equal(dC.cpu().numpy(), want), (ta, tb)


# ------------------------------------------------------------------ bf16 with bias (config 2 shape family)

def _bf16_problem(m, n, k, seed):
    rng = np.random.default_rng(seed)
    A = oracle.round_to("bf16", (rng.standard_normal(m * k) / np.sqrt(k)).astype(np.float32))
    B = oracle.round_to("bf16", (rng.standard_normal(k * n) / np.sqrt(k)).astype(np.float32))
    bias = (rng.standard_normal(n) * 0.02).astype(np.float32)
    return A, B, bias


@pytest.mark.parametrize("ta,tb", [(1, 0), (0, 0), (0, 1), (1, 1)])
@pytest.mark.parametrize("shape", [(512, 768, 320), (300, 520, 200), (1024, 1024, 1024)])
def test_gemmex_bf16_bias(blas, ta, tb, shape):
    m, n, k = shape
    A, B, bias = _bf16_problem(m, n, k, 7)
    lda, ldb = (k if ta else m), (n if tb else k)
    want = oracle.gemm_f64(ta, tb, m, n, k, 1.0, A, lda, B, ldb, bias=bias)
    dC = torch.full((m * n,), float("nan"), dtype=torch.bfloat16, device="cuda")
    dbias = dev_f32(bias)
    assert blas.set_epilogue(bias=dbias, bias_type=N.GRX_R_32F) == N.SUCCESS
    st = blas.gemm_ex(ta, tb, m, n, k, 1.0, dev_bits(oracle.encode("bf16", A)), N.GRX_R_16BF, lda,
                      dev_bits(oracle.encode("bf16", B)), N.GRX_R_16BF, ldb, 0.0, dC, N.GRX_R_16BF, m)
    assert st == N.SUCCESS
    torch.cuda.synchronize()
    assert blas.execution_status() == N.SUCCESS
    ok, nbad = close(dC.float().cpu().numpy(), want)
    assert ok, f"{nbad} elements out of tolerance"


def test_gemmex_bf16_8192_sampled(blas):
    """BASELINE config 2 at full size (8192^3 + bias, bf16 out): 24 full columns
    (first, last and random) checked against the fp64 oracle."""
    m = n = k = 8192
    g = torch.Generator(device="cuda").manual_seed(11)
    dA = (torch.randn(k, m, device="cuda", generator=g) / k ** 0.5).to(torch.bfloat16)  # stored k x m (OP_T)
    dB = (torch.randn(n, k, device="cuda", generator=g) / k ** 0.5).to(torch.bfloat16)  # stored k x n col-major
    dbias = torch.randn(n, device="cuda", generator=g) * 0.02
    dC = torch.empty(n, m, dtype=torch.bfloat16, device="cuda")  # column-major m x n
    assert blas.set_epilogue(bias=dbias, bias_type=N.GRX_R_32F) == N.SUCCESS
    st = blas.gemm_ex(1, 0, m, n, k, 1.0, dA, N.GRX_R_16BF, k, dB, N.GRX_R_16BF, k, 0.0, dC, N.GRX_R_16BF, m)
    assert st == N.SUCCESS
    torch.cuda.synchronize()
    assert blas.execution_status() == N.SUCCESS
    cols = np.unique(np.concatenate([[0, 1, 255, 256, n - 1], np.random.default_rng(3).integers(0, n, 19)]))
    A = dA.float().cpu().numpy().ravel()
    Bsub = dB[torch.as_tensor(cols, device="cuda")].float().cpu().numpy().ravel()  # len(cols) x k
    want = oracle.gemm_f64(1, 0, m, len(cols), k, 1.0, A, k, Bsub, k, bias=dbias.cpu().numpy()[cols])
    got = dC[torch.as_tensor(cols, device="cuda")].float().cpu().numpy().ravel()
    ok, nbad = close(got, want)
    assert ok, f"{nbad} of {got.size} out of tolerance"


# ------------------------------------------------------------------ fp8 and scaled int8 (config 5 family)

def test_gemm_fp8_per_tensor_scale_batched(blas):
    batch, m, n, k = 3, 320, 448, 512
    rng = np.random.default_rng(21)
    Af = rng.standard_normal((batch, k, m)).astype(np.float32)  # OP_T: stored k x m
    Bf = rng.standard_normal((batch, n, k)).astype(np.float32)  # OP_N: stored k x n column-major
    sa = (np.abs(Af).reshape(batch, -1).max(1) / 448).astype(np.float32)
    sb = (np.abs(Bf).reshape(batch, -1).max(1) / 448).astype(np.float32)
    Aq = oracle.encode("e4m3", Af / sa[:, None, None])
    Bq = oracle.encode("e4m3", Bf / sb[:, None, None])
    Ad, Bd = oracle.decode("e4m3", Aq).ravel(), oracle.decode("e4m3", Bq).ravel()
    want = oracle.gemm_f64(1, 0, m, n, k, 1.0, Ad, k, Bd, k, sA=k * m, sB=k * n, sC=m * n, batch=batch,
                           scale_mode=1, sa=sa, sb=sb, ssa=1, ssb=1)
    dC = torch.full((batch * m * n,), float("nan"), dtype=torch.bfloat16, device="cuda")
    dsa, dsb = dev_f32(sa), dev_f32(sb)  # the handle keeps the pointers, not the tensors
    assert blas.set_epilogue(scale_mode=N.SCALE_TENSOR, scale_a=dsa, scale_b=dsb,
                             stride_scale_a=1, stride_scale_b=1) == N.SUCCESS
    st = blas.gemm_strided_batched_ex(1, 0, m, n, k, 1.0, dev_bits(Aq), N.GRX_R_8F_E4M3, k, k * m, dev_bits(Bq),
                                      N.GRX_R_8F_E4M3, k, k * n, 0.0, dC, N.GRX_R_16BF, m, m * n, batch)
    assert st == N.SUCCESS
    torch.cuda.synchronize()
    ok, nbad = close(dC.float().cpu().numpy(), want)
    assert ok, nbad


def test_gemm_int8_rowcol_scale(blas):
    m, n, k = 384, 520, 640
    rng = np.random.default_rng(23)
    Af = rng.standard_normal((m, k)).astype(np.float32)  # rows of op(A)
    Bf = rng.standard_normal((n, k)).astype(np.float32)  # columns of op(B), k contiguous
    sa = (np.abs(Af).max(1) / 127).astype(np.float32)
    sb = (np.abs(Bf).max(1) / 127).astype(np.float32)
    Aq = np.clip(np.rint(Af / sa[:, None]), -127, 127).astype(np.int8)  # stored k x m (OP_T): row i contiguous in k
    Bq = np.clip(np.rint(Bf / sb[:, None]), -127, 127).astype(np.int8)  # stored k x n (OP_N)
    want = oracle.gemm_f64(1, 0, m, n, k, 1.0, Aq.astype(np.float32).ravel(), k, Bq.astype(np.float32).ravel(), k,
                           scale_mode=2, sa=sa, sb=sb)
    dC = torch.full((m * n,), float("nan"), dtype=torch.bfloat16, device="cuda")
    dsa, dsb = dev_f32(sa), dev_f32(sb)  # the handle keeps the pointers, not the tensors
    assert blas.set_epilogue(scale_mode=N.SCALE_ROWCOL, scale_a=dsa, scale_b=dsb) == N.SUCCESS
    st = blas.gemm_ex(1, 0, m, n, k, 1.0, dev_bits(Aq.ravel()), N.GRX_R_8I, k, dev_bits(Bq.ravel()), N.GRX_R_8I, k,
                      0.0, dC, N.GRX_R_16BF, m)
    assert st == N.SUCCESS
    torch.cuda.synchronize()
    ok, nbad = close(dC.float().cpu().numpy(), want)
    assert ok, nbad


def test_gemmex_strided_batched_bf16_broadcast_and_slack(blas):
    batch, m, n, k, gap = 4, 136, 264, 72, 8
    rng = np.random.default_rng(9)
    sa, sc = m * k + gap, m * n + gap
    A = oracle.round_to("bf16", rng.standard_normal(sa * batch).astype(np.float32))
    B = oracle.round_to("bf16", rng.standard_normal(k * n).astype(np.float32))  # broadcast, strideB = 0
    C = oracle.round_to("bf16", rng.standard_normal(sc * batch).astype(np.float32))
    want = C.astype(np.float64).copy()
    for bi in range(batch):
        part = oracle.gemm_f64(0, 0, m, n, k, 1.5, A[sa * bi:], m, B, k, beta=-0.5,
                               Cin=C[sc * bi:sc * bi + m * n].astype(np.float64), ldc=m)
        want[sc * bi:sc * bi + m * n] = part
    dC = dev_bits(oracle.encode("bf16", C))
    st = blas.gemm_strided_batched_ex(0, 0, m, n, k, 1.5, dev_bits(oracle.encode("bf16", A)), N.GRX_R_16BF, m, sa,
                                      dev_bits(oracle.encode("bf16", B)), N.GRX_R_16BF, k, 0, -0.5, dC,
                                      N.GRX_R_16BF, m, sc, batch)
    assert st == N.SUCCESS
    torch.cuda.synchronize()
    got = oracle.decode("bf16", dC.cpu().numpy().view(np.uint16))
    ok, nbad = close(got, want)
    assert ok, nbad
    # the slack between batch members is untouched
    for bi in range(batch):
        s = sc * bi + m * n
        assert np.array_equal(got[s:s + gap], C[s:s + gap].astype(np.float32))


def test_gemm_refusals_on_device(blas):
    d = torch.zeros(4096, dtype=torch.uint8, device="cuda")
    one = 1.0
    # fp32 input refused (test_grxblas_ex.cpp:353-357)
    assert blas.gemm_ex(0, 0, 8, 4, 8, one, d, N.GRX_R_32F, 8, d, N.GRX_R_16F, 8, 0.0, d, N.GRX_R_32F, 8) == \
        N.NOT_SUPPORTED
    # non-integral alpha on the int8 pairing (test_grxblas_ex.cpp:334-341)
    assert blas.gemm_ex(0, 0, 8, 4, 16, 2.5, d, N.GRX_R_8I, 8, d, N.GRX_R_8I, 16, 0.0, d, N.GRX_R_32I, 8) == \
        N.INVALID_VALUE
    # mixed 16-bit input types
    assert blas.gemm_ex(0, 0, 8, 4, 8, one, d, N.GRX_R_16F, 8, d, N.GRX_R_16BF, 8, 0.0, d, N.GRX_R_32F, 8) == \
        N.NOT_SUPPORTED


# ------------------------------------------------------------------ CTA-pair path (forced for every type)

@pytest.mark.parametrize("ta,tb", [(1, 0), (0, 0), (0, 1), (1, 1)])
def test_pair_path_bf16_bias_ragged(blas, ta, tb, monkeypatch):
    monkeypatch.setenv("GRX_GEMM_FORCE_PAIR", "1")
    """Problems large enough for the cta_group::2 kernel (256 x 256 tiles over CTA pairs),
    every transpose, ragged m and n (edge tiles of both CTAs of a pair)."""
    m, n, k = 2600, 2100, 320
    A, B, bias = _bf16_problem(m, n, k, 17)
    lda, ldb = (k if ta else m), (n if tb else k)
    want = oracle.gemm_f64(ta, tb, m, n, k, 1.0, A, lda, B, ldb, bias=bias)
    dC = torch.full((m * n,), float("nan"), dtype=torch.bfloat16, device="cuda")
    dbias = dev_f32(bias)
    assert blas.set_epilogue(bias=dbias, bias_type=N.GRX_R_32F) == N.SUCCESS
    st = blas.gemm_ex(ta, tb, m, n, k, 1.0, dev_bits(oracle.encode("bf16", A)), N.GRX_R_16BF, lda,
                      dev_bits(oracle.encode("bf16", B)), N.GRX_R_16BF, ldb, 0.0, dC, N.GRX_R_16BF, m)
    assert st == N.SUCCESS
    torch.cuda.synchronize()
    assert blas.execution_status() == N.SUCCESS
    ok, nbad = close(dC.float().cpu().numpy(), want)
    assert ok, f"{nbad} elements out of tolerance"


@pytest.mark.parametrize("ta,tb", [(1, 0), (0, 1)])
def test_pair_path_int8_exact_with_beta(blas, ta, tb, monkeypatch):
    monkeypatch.setenv("GRX_GEMM_FORCE_PAIR", "1")
    m, n, k, pad = 2560, 2048, 256, 16
    a_rows, a_cols = (k, m) if ta else (m, k)
    b_rows, b_cols = (n, k) if tb else (k, n)
    lda, ldb, ldc = a_rows + pad, b_rows + pad, m + pad
    A, B, C = int8_patterns(lda * a_cols, ldb * b_cols, ldc * n)
    want = oracle.igemm(ta, tb, m, n, k, 3, A, lda, B, ldb, -2, C, ldc)
    dC = torch.from_numpy(C.copy()).cuda()
    st = blas.gemm_ex(ta, tb, m, n, k, 3.0, dev_bits(A), N.GRX_R_8I, lda, dev_bits(B), N.GRX_R_8I, ldb, -2.0, dC,
                      N.GRX_R_32I, ldc)
    assert st == N.SUCCESS
    torch.cuda.synchronize()
    assert np.array_equal(dC.cpu().numpy(), want)


def test_pair_path_fp8_batched_scaled(blas, monkeypatch):
    monkeypatch.setenv("GRX_GEMM_FORCE_PAIR", "1")
    batch, m, n, k = 4, 1024, 1536, 384
    rng = np.random.default_rng(29)
    Af = rng.standard_normal((batch, m, k)).astype(np.float32)  # OP_T: stored k x m
    Bf = rng.standard_normal((batch, n, k)).astype(np.float32)
    sa = (np.abs(Af).reshape(batch, -1).max(1) / 448).astype(np.float32)
    sb = (np.abs(Bf).reshape(batch, -1).max(1) / 448).astype(np.float32)
    Aq = oracle.encode("e4m3", Af / sa[:, None, None])
    Bq = oracle.encode("e4m3", Bf / sb[:, None, None])
    want = oracle.gemm_f64(1, 0, m, n, k, 1.0, oracle.decode("e4m3", Aq).ravel(), k,
                           oracle.decode("e4m3", Bq).ravel(), k, sA=k * m, sB=k * n, sC=m * n, batch=batch,
                           scale_mode=1, sa=sa, sb=sb, ssa=1, ssb=1)
    dC = torch.full((batch * m * n,), float("nan"), dtype=torch.bfloat16, device="cuda")
    dsa, dsb = dev_f32(sa), dev_f32(sb)
    assert blas.set_epilogue(scale_mode=N.SCALE_TENSOR, scale_a=dsa, scale_b=dsb, stride_scale_a=1,
                             stride_scale_b=1) == N.SUCCESS
    st = blas.gemm_strided_batched_ex(1, 0, m, n, k, 1.0, dev_bits(Aq), N.GRX_R_8F_E4M3, k, k * m, dev_bits(Bq),
                                      N.GRX_R_8F_E4M3, k, k * n, 0.0, dC, N.GRX_R_16BF, m, m * n, batch)
    assert st == N.SUCCESS
    torch.cuda.synchronize()
    ok, nbad = close(dC.float().cpu().numpy(), want)
    assert ok, nbad


# ------------------------------------------------------------------ epilogue: row bias and activations

@pytest.mark.parametrize("act", [N.ACT_RELU, N.ACT_GELU_TANH, N.ACT_GELU_ERF])
@pytest.mark.parametrize("rows", [False, True])
def test_epilogue_bias_activation(blas, act, rows):
    m, n, k = 384, 520, 256
    A, B, _ = _bf16_problem(m, n, k, 31)
    bias = (np.random.default_rng(2).standard_normal(m if rows else n) * 0.5).astype(np.float32)
    lin = oracle.gemm_f64(1, 0, m, n, k, 1.0, A, k, B, k).reshape(n, m).T
    lin = lin + (bias[:, None] if rows else bias[None, :])
    if act == N.ACT_RELU:
        want = np.maximum(lin, 0)
    else:
        want = oracle.gelu(lin.astype(np.float32), 0 if act == N.ACT_GELU_ERF else 1)
    dC = torch.full((m * n,), float("nan"), dtype=torch.bfloat16, device="cuda")
    dbias = dev_f32(bias)
    assert blas.set_epilogue(bias=dbias, bias_type=N.GRX_R_32F, bias_over_rows=rows, activation=act) == N.SUCCESS
    assert blas.gemm_ex(1, 0, m, n, k, 1.0, dev_bits(oracle.encode("bf16", A)), N.GRX_R_16BF, k,
                        dev_bits(oracle.encode("bf16", B)), N.GRX_R_16BF, k, 0.0, dC, N.GRX_R_16BF, m) == N.SUCCESS
    torch.cuda.synchronize()
    got = dC.float().cpu().numpy().reshape(n, m).T
    ok, nbad = close(got, want)
    assert ok, nbad


def test_epilogue_activation_refused_for_exact_int8(blas):
    d = torch.zeros(4096, dtype=torch.int8, device="cuda")
    c = torch.zeros(1024, dtype=torch.int32, device="cuda")
    assert blas.set_epilogue(activation=N.ACT_RELU) == N.SUCCESS
    assert blas.gemm_ex(0, 0, 8, 4, 16, 1.0, d, N.GRX_R_8I, 8, d, N.GRX_R_8I, 16, 0.0, c, N.GRX_R_32I, 8) == \
        N.NOT_SUPPORTED
    assert blas.set_epilogue(activation=9) == N.INVALID_VALUE


# ------------------------------------------------------------------ config 5 at full size

def _quantize_e4m3_per_tensor(x):
    """x [batch, rows, k] fp32 -> (e4m3 codes, per-batch-member scale amax / 448)."""
    amax = x.abs().amax(dim=(1, 2)).clamp_min(1e-30)
    scale = (amax / 448.0).float()
    return (x / scale[:, None, None]).to(torch.float8_e4m3fn), scale


def _config5_columns(n, batch_member):
    rng = np.random.default_rng(100 + batch_member)
    return np.unique(np.concatenate([[0, 1, 255, 256, n - 1], rng.integers(0, n, 11)]))


@pytest.mark.parametrize("kind", ["fp8_per_tensor", "int8_rowcol"])
def test_config5_full_size_sampled(blas, kind):
    """BASELINE config 5 at its real size: batch 16 x M=4096 x N=14336 x K=4096,
    A/B ~ N(0,1) quantised (e4m3 with per-tensor amax/448 scales, or int8 with
    per-row / per-column amax/127 scales), fp32 accumulate, bf16 out through the
    fused scale epilogue. 16 full output columns (first, last, tile seams, random)
    of batch members 0, 7 and 15 are checked against the fp64 oracle of the
    dequantised inputs within 1e-2 + 2e-2 |ref|."""
    bt, m, n, k = 16, 4096, 14336, 4096
    g = torch.Generator(device="cuda").manual_seed(55)
    af = torch.randn(bt, m, k, device="cuda", generator=g)
    if kind == "fp8_per_tensor":
        a8, sa = _quantize_e4m3_per_tensor(af)
        del af
        bf = torch.randn(bt, n, k, device="cuda", generator=g)
        b8, sb = _quantize_e4m3_per_tensor(bf)
        del bf
        atype = N.GRX_R_8F_E4M3
        assert blas.set_epilogue(scale_mode=N.SCALE_TENSOR, scale_a=sa, scale_b=sb, stride_scale_a=1,
                                 stride_scale_b=1) == N.SUCCESS
    else:
        # per-row scales of op(A) and per-column of op(B), shared by the batch (stride 0)
        sa = (af.abs().amax(dim=(0, 2)) / 127).clamp_min(1e-30)
        a8 = torch.clamp(torch.round(af / sa[None, :, None]), -127, 127).to(torch.int8)
        del af
        bf = torch.randn(bt, n, k, device="cuda", generator=g)
        sb = (bf.abs().amax(dim=(0, 2)) / 127).clamp_min(1e-30)
        b8 = torch.clamp(torch.round(bf / sb[None, :, None]), -127, 127).to(torch.int8)
        del bf
        atype = N.GRX_R_8I
        assert blas.set_epilogue(scale_mode=N.SCALE_ROWCOL, scale_a=sa, scale_b=sb) == N.SUCCESS
    c = torch.empty(bt, n, m, device="cuda", dtype=torch.bfloat16)
    st = blas.gemm_strided_batched_ex(1, 0, m, n, k, 1.0, a8, atype, k, m * k, b8, atype, k, n * k, 0.0, c,
                                      N.GRX_R_16BF, m, m * n, bt)
    assert st == N.SUCCESS
    torch.cuda.synchronize()
    assert blas.execution_status() == N.SUCCESS
    blas.clear_epilogue()
    for bi in (0, 7, 15):
        cols = _config5_columns(n, bi)
        idx = torch.as_tensor(cols, device="cuda")
        A = a8[bi].float().cpu().numpy().ravel()  # codes as values (e4m3 decodes exactly to fp32)
        Bsub = b8[bi][idx].float().cpu().numpy().ravel()
        if kind == "fp8_per_tensor":
            want = oracle.gemm_f64(1, 0, m, len(cols), k, 1.0, A, k, Bsub, k, scale_mode=1,
                                   sa=sa[bi:bi + 1].cpu().numpy(), sb=sb[bi:bi + 1].cpu().numpy())
        else:
            want = oracle.gemm_f64(1, 0, m, len(cols), k, 1.0, A, k, Bsub, k, scale_mode=2, sa=sa.cpu().numpy(),
                                   sb=sb[idx].cpu().numpy())
        got = c[bi][idx].float().cpu().numpy().ravel()
        ok, nbad = close(got, want)
        assert ok, f"batch {bi}: {nbad} of {got.size} out of tolerance"
    del a8, b8, c
    torch.cuda.empty_cache()
