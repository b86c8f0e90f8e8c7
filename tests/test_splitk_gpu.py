"""GPU parity of the split-K tail schedule (tiles cut into k-ranges that run
as separate units on different CTAs).

The schedule only changes which unit accumulates which k-blocks of a tile
and how the cut tiles' partial sums are combined, so every gate of the
whole-tile kernel applies unchanged: int8 -> int32 bit-exact against the
oracle, bf16 / fp8 within |got - ref| <= 1e-2 + 2e-2*|ref| of the fp64 oracle,
no write outside the m x n window. GRX_GEMM_FORCE_SK=s cuts every tile into s
k-ranges, so modest problems exercise 2..8 pieces per tile; one case checks
the automatic plan (a tile count just past one wave of SMs) and one checks
from the GRXPROF trace that the forced launch really ran tiles x s units."""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

import oracle
from gates import int8_patterns
from grxcp_b200 import _native as N

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parent.parent
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


def close(got, ref):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    bad = np.abs(got - ref) > TOL_ABS + TOL_REL * np.abs(ref)
    return not bad.any(), int(bad.sum())


def bf16_problem(m, n, k, seed):
    rng = np.random.default_rng(seed)
    A = oracle.round_to("bf16", (rng.standard_normal(m * k) / np.sqrt(k)).astype(np.float32))
    B = oracle.round_to("bf16", (rng.standard_normal(k * n) / np.sqrt(k)).astype(np.float32))
    bias = (rng.standard_normal(n) * 0.1).astype(np.float32)
    return A, B, bias


@pytest.mark.parametrize("splits", [2, 5, 8])
@pytest.mark.parametrize("ta,tb", [(1, 0), (0, 1)])
def test_splitk_int8_exact_with_beta(blas, splits, ta, tb, monkeypatch):
    """15 tiles of 32 k-blocks, each cut into `splits` ranges: integer
    partials summed exactly; ld padding of C untouched."""
    monkeypatch.setenv("GRX_GEMM_FORCE_SK", str(splits))
    m, n, k, pad = 600, 700, 4096, 8
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
    assert blas.execution_status() == N.SUCCESS
    assert np.array_equal(dC.cpu().numpy(), want)


@pytest.mark.parametrize("splits", [3, 8])
@pytest.mark.parametrize("out", ["bf16", "f32"])
def test_splitk_bf16_bias_gelu_ragged(blas, splits, out, monkeypatch):
    """Ragged edge tiles, column bias and a GELU epilogue applied once, after
    the pieces are summed (applying it per piece would be wrong)."""
    monkeypatch.setenv("GRX_GEMM_FORCE_SK", str(splits))
    m, n, k = 333, 517, 1000
    A, B, bias = bf16_problem(m, n, k, 41)
    lin = oracle.gemm_f64(1, 0, m, n, k, 1.0, A, k, B, k).reshape(n, m).T + bias[None, :]
    want = oracle.gelu(lin.astype(np.float32), 1)
    ct = N.GRX_R_16BF if out == "bf16" else N.GRX_R_32F
    dC = torch.full((m * n,), float("nan"), dtype=torch.bfloat16 if out == "bf16" else torch.float32, device="cuda")
    dbias = dev_f32(bias)
    assert blas.set_epilogue(bias=dbias, bias_type=N.GRX_R_32F, activation=N.ACT_GELU_TANH) == N.SUCCESS
    st = blas.gemm_ex(1, 0, m, n, k, 1.0, dev_bits(oracle.encode("bf16", A)), N.GRX_R_16BF, k,
                      dev_bits(oracle.encode("bf16", B)), N.GRX_R_16BF, k, 0.0, dC, ct, m)
    assert st == N.SUCCESS
    torch.cuda.synchronize()
    assert blas.execution_status() == N.SUCCESS
    got = dC.float().cpu().numpy().reshape(n, m).T
    ok, nbad = close(got, want)
    assert ok, f"{nbad} elements out of tolerance"


def test_splitk_bf16_beta_reads_c_once(blas, monkeypatch):
    """beta != 0: C is read by the reducing warp only, so beta*C is added once."""
    monkeypatch.setenv("GRX_GEMM_FORCE_SK", "3")
    m, n, k = 256, 512, 2048
    A, B, _ = bf16_problem(m, n, k, 5)
    C0 = np.random.default_rng(6).standard_normal(m * n).astype(np.float32)
    want = oracle.gemm_f64(0, 1, m, n, k, 0.5, A, m, B, n, beta=-1.5, Cin=C0)
    dC = dev_f32(C0)
    st = blas.gemm_ex(0, 1, m, n, k, 0.5, dev_bits(oracle.encode("bf16", A)), N.GRX_R_16BF, m,
                      dev_bits(oracle.encode("bf16", B)), N.GRX_R_16BF, n, -1.5, dC, N.GRX_R_32F, m)
    assert st == N.SUCCESS
    torch.cuda.synchronize()
    ok, nbad = close(dC.cpu().numpy(), want)
    assert ok, nbad


def test_splitk_fp8_batched_per_channel_scales(blas, monkeypatch):
    """Cut tiles of several batch members (12 k-blocks in 5 uneven ranges)."""
    monkeypatch.setenv("GRX_GEMM_FORCE_SK", "5")
    batch, m, n, k = 3, 256, 384, 1536
    rng = np.random.default_rng(8)
    Af = rng.standard_normal((batch, m, k)).astype(np.float32)
    Bf = rng.standard_normal((batch, n, k)).astype(np.float32)
    sa = (np.abs(Af).max(2) / 448).astype(np.float32)  # per row of each member
    sb = (np.abs(Bf).max(2) / 448).astype(np.float32)  # per column
    Aq = oracle.encode("e4m3", Af / sa[:, :, None])
    Bq = oracle.encode("e4m3", Bf / sb[:, :, None])
    want = oracle.gemm_f64(1, 0, m, n, k, 1.0, oracle.decode("e4m3", Aq).ravel(), k,
                           oracle.decode("e4m3", Bq).ravel(), k, sA=k * m, sB=k * n, sC=m * n, batch=batch,
                           scale_mode=2, sa=sa.ravel(), sb=sb.ravel(), ssa=m, ssb=n)
    dC = torch.full((batch * m * n,), float("nan"), dtype=torch.bfloat16, device="cuda")
    dsa, dsb = dev_f32(sa.ravel()), dev_f32(sb.ravel())
    assert blas.set_epilogue(scale_mode=N.SCALE_ROWCOL, scale_a=dsa, scale_b=dsb, stride_scale_a=m,
                             stride_scale_b=n) == N.SUCCESS
    st = blas.gemm_strided_batched_ex(1, 0, m, n, k, 1.0, dev_bits(Aq), N.GRX_R_8F_E4M3, k, k * m, dev_bits(Bq),
                                      N.GRX_R_8F_E4M3, k, k * n, 0.0, dC, N.GRX_R_16BF, m, m * n, batch)
    assert st == N.SUCCESS
    torch.cuda.synchronize()
    ok, nbad = close(dC.float().cpu().numpy(), want)
    assert ok, nbad


def test_splitk_automatic_plan_long_k(blas, monkeypatch):
    """No forcing: 1024 x 1024 x 8192 is 32 tiles of 128 k-blocks, far less
    than one wave of SMs, which the automatic plan cuts; checked twice, the
    second call reusing the workspace and its arrival counters."""
    monkeypatch.delenv("GRX_GEMM_FORCE_SK", raising=False)
    m, n, k = 1024, 1024, 8192
    A, B, bias = bf16_problem(m, n, k, 12)
    want = oracle.gemm_f64(1, 0, m, n, k, 1.0, A, k, B, k, bias=bias)
    dC = torch.full((m * n,), float("nan"), dtype=torch.bfloat16, device="cuda")
    dbias = dev_f32(bias)
    assert blas.set_epilogue(bias=dbias, bias_type=N.GRX_R_32F) == N.SUCCESS
    for _ in range(2):
        st = blas.gemm_ex(1, 0, m, n, k, 1.0, dev_bits(oracle.encode("bf16", A)), N.GRX_R_16BF, k,
                          dev_bits(oracle.encode("bf16", B)), N.GRX_R_16BF, k, 0.0, dC, N.GRX_R_16BF, m)
        assert st == N.SUCCESS
        torch.cuda.synchronize()
        assert blas.execution_status() == N.SUCCESS
        ok, nbad = close(dC.float().cpu().numpy(), want)
        assert ok, nbad


CHILD = r"""
import sys; sys.path.insert(0, %r)
import torch
from grxcp_b200 import blas as B, _native as N
a = torch.randn(700 * 2048, device="cuda").to(torch.bfloat16)
c = torch.empty(600 * 700, device="cuda", dtype=torch.bfloat16)
with B.Handle() as h:
    assert h.gemm_ex(1, 0, 600, 700, 2048, 1.0, a, N.GRX_R_16BF, 2048, a, N.GRX_R_16BF, 2048, 0.0, c,
                     N.GRX_R_16BF, 600) == 0
    torch.cuda.synchronize()
    assert h.execution_status() == 0
""" % str(ROOT)


def test_forced_schedule_runs_every_range_as_a_unit():
    env = dict(os.environ, GRX_PROFILE="1", GRX_GEMM_FORCE_SK="3")
    r = subprocess.run([sys.executable, "-c", CHILD], env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    grids = [dict(f.split("=", 1) for f in l.split("|")[2:])["grid"] for l in r.stderr.splitlines()
             if l.startswith("GRXPROF|1|op=launch|") and "kernel=tc_gemm_kernel" in l]
    assert grids == ["45.1.1"], grids  # 15 tiles x 3 ranges; whole tiles would launch 15 CTAs


# ------------------------------------------------------------------ the CTA-pair kernel's split-K tail

@pytest.mark.parametrize("splits", [2, 5])
@pytest.mark.parametrize("ta,tb", [(1, 0), (0, 1)])
def test_pair_splitk_int8_exact_with_beta(blas, splits, ta, tb, monkeypatch):
    """The pair kernel with every 256 x 256 tile cut into `splits` k-ranges:
    each CTA of a pair publishes its own 128-row half; integer partials summed
    exactly in split order; ld padding of C untouched."""
    monkeypatch.setenv("GRX_GEMM_FORCE_PAIR", "1")
    monkeypatch.setenv("GRX_GEMM_FORCE_SK", str(splits))
    m, n, k, pad = 600, 700, 4096, 8
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
    assert blas.execution_status() == N.SUCCESS
    assert np.array_equal(dC.cpu().numpy(), want)


@pytest.mark.parametrize("splits", [3, 8])
def test_pair_splitk_bf16_bias_gelu_ragged(blas, splits, monkeypatch):
    monkeypatch.setenv("GRX_GEMM_FORCE_PAIR", "1")
    monkeypatch.setenv("GRX_GEMM_FORCE_SK", str(splits))
    m, n, k = 333, 517, 1000
    A, B, bias = bf16_problem(m, n, k, 43)
    lin = oracle.gemm_f64(1, 0, m, n, k, 1.0, A, k, B, k).reshape(n, m).T + bias[None, :]
    want = oracle.gelu(lin.astype(np.float32), 1)
    dC = torch.full((m * n,), float("nan"), dtype=torch.bfloat16, device="cuda")
    dbias = dev_f32(bias)
    assert blas.set_epilogue(bias=dbias, bias_type=N.GRX_R_32F, activation=N.ACT_GELU_TANH) == N.SUCCESS
    st = blas.gemm_ex(1, 0, m, n, k, 1.0, dev_bits(oracle.encode("bf16", A)), N.GRX_R_16BF, k,
                      dev_bits(oracle.encode("bf16", B)), N.GRX_R_16BF, k, 0.0, dC, N.GRX_R_16BF, m)
    assert st == N.SUCCESS
    torch.cuda.synchronize()
    assert blas.execution_status() == N.SUCCESS
    ok, nbad = close(dC.float().cpu().numpy().reshape(n, m).T, want)
    assert ok, f"{nbad} elements out of tolerance"


def test_pair_splitk_automatic_plan_on_the_four_gpu_slice(blas):
    """8192 x 2048 x 8192 bf16 + bias (one rank's slice at 4 GPUs): 256 pair
    tiles on 74 SM pairs, whose last partial round the planner cuts in two.
    Sampled full columns (first, last, tile seams, random) against the fp64
    oracle; a repeat call is bit-identical (deterministic reduction)."""
    m, n, k = 8192, 2048, 8192
    g = torch.Generator(device="cuda").manual_seed(12)
    dA = (torch.randn(k, m, device="cuda", generator=g) / k ** 0.5).to(torch.bfloat16)
    dB = (torch.randn(n, k, device="cuda", generator=g) / k ** 0.5).to(torch.bfloat16)
    dbias = torch.randn(n, device="cuda", generator=g) * 0.02
    dC = torch.empty(n, m, dtype=torch.bfloat16, device="cuda")
    assert blas.set_epilogue(bias=dbias, bias_type=N.GRX_R_32F) == N.SUCCESS
    call = lambda c: blas.gemm_ex(1, 0, m, n, k, 1.0, dA, N.GRX_R_16BF, k, dB, N.GRX_R_16BF, k, 0.0, c,  # noqa: E731
                                  N.GRX_R_16BF, m)
    assert call(dC) == N.SUCCESS
    dC2 = torch.empty_like(dC)
    assert call(dC2) == N.SUCCESS
    torch.cuda.synchronize()
    assert blas.execution_status() == N.SUCCESS
    assert torch.equal(dC, dC2)
    cols = np.unique(np.concatenate([[0, 1, 255, 256, 1791, 1792, n - 1], np.random.default_rng(4).integers(0, n, 9)]))
    A = dA.float().cpu().numpy().ravel()
    Bsub = dB[torch.as_tensor(cols, device="cuda")].float().cpu().numpy().ravel()
    want = oracle.gemm_f64(1, 0, m, len(cols), k, 1.0, A, k, Bsub, k, bias=dbias.cpu().numpy()[cols])
    got = dC[torch.as_tensor(cols, device="cuda")].float().cpu().numpy().ravel()
    ok, nbad = close(got, want)
    assert ok, f"{nbad} of {got.size} out of tolerance"
