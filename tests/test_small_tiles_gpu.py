"""GPU parity of the single-CTA kernel's narrow tiles. A problem whose
128 x 256 tiles would fill at most half the SMs (and that takes no split-K
tail) runs with the tile's columns halved until the tiles would outnumber
the SMs (down to 128 x 32; an MN-major B keeps whole 128-byte atoms), so
more SMs share the MMAs and the epilogue's stores -- BASELINE config 1's
int8 512^3 runs 64 CTAs instead of 8.

Only the output tiling changes, so the gates of the wide kernel apply to
both tilings (GRX_GEMM_WIDE_TILES=1 forces 128 x 256): int8 -> int32 exact,
bf16/fp8 within 1e-2 + 2e-2*|ref| of the fp64 oracle, nothing written
outside m x n; and since each output element sums the same k-steps in the
same order either way, the two tilings agree bit for bit."""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

import oracle
from grxcp_b200 import _native as N

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parent.parent
TOL_ABS, TOL_REL = 1e-2, 2e-2


def dev_bits(bits):
    b = np.ascontiguousarray(bits)
    if b.dtype == np.uint16:
        return torch.from_numpy(b.view(np.int16)).cuda()
    if b.dtype == np.uint8:
        return torch.from_numpy(b.view(np.int8)).cuda()
    return torch.from_numpy(b).cuda()


def both(call, monkeypatch):
    """Runs call() with narrow tiles, then with 128 x 256 tiles."""
    narrow = call()
    monkeypatch.setenv("GRX_GEMM_WIDE_TILES", "1")
    wide = call()
    monkeypatch.delenv("GRX_GEMM_WIDE_TILES")
    return narrow, wide


@pytest.mark.parametrize("ta,tb", [(0, 0), (1, 0), (0, 1), (1, 1)])
def test_int8_512_config1_exact(blas, ta, tb, monkeypatch):
    m = n = k = 512
    rng = np.random.default_rng(40 + 2 * ta + tb)
    A = rng.integers(-128, 128, m * k).astype(np.int8)
    B = rng.integers(-128, 128, k * n).astype(np.int8)
    C0 = np.zeros(m * n, np.int32)
    want = oracle.igemm(ta, tb, m, n, k, 1, A, 512, B, 512, 0, C0, m)

    def call():
        dC = torch.full((m * n,), 12345, dtype=torch.int32, device="cuda")
        assert blas.gemm_ex(ta, tb, m, n, k, 1.0, dev_bits(A), N.GRX_R_8I, 512, dev_bits(B), N.GRX_R_8I, 512, 0.0,
                            dC, N.GRX_R_32I, m) == N.SUCCESS
        torch.cuda.synchronize()
        assert blas.execution_status() == N.SUCCESS
        return dC.cpu().numpy()

    narrow, wide = both(call, monkeypatch)
    assert np.array_equal(narrow, want)
    assert np.array_equal(wide, want)


@pytest.mark.parametrize("m,n,k", [(300, 520, 200), (512, 96, 1024), (128, 40, 64), (1000, 333, 256)])
@pytest.mark.parametrize("ta,tb", [(1, 0), (0, 1)])
def test_bf16_bias_narrow_and_wide(blas, m, n, k, ta, tb, monkeypatch):
    pad = 6
    rng = np.random.default_rng(m * 7 + n + k)
    a_rows, a_cols = (k, m) if ta else (m, k)
    b_rows, b_cols = (n, k) if tb else (k, n)
    lda, ldb, ldc = a_rows, b_rows, m + pad
    A = oracle.round_to("bf16", (rng.standard_normal(lda * a_cols) / np.sqrt(k)).astype(np.float32))
    B = oracle.round_to("bf16", (rng.standard_normal(ldb * b_cols) / np.sqrt(k)).astype(np.float32))
    bias = (rng.standard_normal(n) * 0.05).astype(np.float32)
    dA, dB = dev_bits(oracle.encode("bf16", A)), dev_bits(oracle.encode("bf16", B))
    dbias = torch.from_numpy(bias).cuda()  # the handle keeps the pointer: keep the tensor alive
    assert blas.set_epilogue(bias=dbias, bias_type=N.GRX_R_32F) == N.SUCCESS

    def call():
        dC = torch.full((n * ldc,), -3.0, device="cuda")
        assert blas.gemm_ex(ta, tb, m, n, k, 1.0, dA, N.GRX_R_16BF, lda, dB, N.GRX_R_16BF, ldb, 0.0, dC,
                            N.GRX_R_32F, ldc) == N.SUCCESS
        torch.cuda.synchronize()
        assert blas.execution_status() == N.SUCCESS
        return dC.cpu().numpy().reshape(n, ldc)

    want = oracle.gemm_f64(ta, tb, m, n, k, 1.0, A, lda, B, ldb, bias=bias).reshape(n, m)
    narrow, wide = both(call, monkeypatch)
    assert np.array_equal(narrow, wide)
    for got in (narrow, wide):
        assert np.all(got[:, m:] == -3.0), "write into ld padding"
        bad = np.abs(got[:, :m] - want) > TOL_ABS + TOL_REL * np.abs(want)
        assert not bad.any(), int(bad.sum())


def test_fp8_rowcol_scale_batched_narrow_and_wide(blas, monkeypatch):
    batch, m, n, k = 2, 256, 200, 512
    rng = np.random.default_rng(77)
    Af = rng.standard_normal((batch, m, k)).astype(np.float32)  # OP_T, lda = k: row i of op(A) is contiguous
    Bf = rng.standard_normal((batch, n, k)).astype(np.float32)
    Aq = oracle.encode("e4m3", Af / (np.abs(Af).max() / 448))
    Bq = oracle.encode("e4m3", Bf / (np.abs(Bf).max() / 448))
    sa = (rng.random((batch, m)) + 0.5).astype(np.float32)
    sb = (rng.random((batch, n)) + 0.5).astype(np.float32)
    dA, dB = dev_bits(Aq.ravel()), dev_bits(Bq.ravel())
    dsa, dsb = torch.from_numpy(sa).cuda(), torch.from_numpy(sb).cuda()  # kept alive for the calls
    assert blas.set_epilogue(scale_a=dsa, scale_b=dsb,
                             scale_mode=N.SCALE_ROWCOL, stride_scale_a=m, stride_scale_b=n) == N.SUCCESS

    def call():
        dC = torch.zeros(batch * n * m, dtype=torch.bfloat16, device="cuda")
        assert blas.gemm_strided_batched_ex(1, 0, m, n, k, 1.0, dA, N.GRX_R_8F_E4M3, k, k * m, dB, N.GRX_R_8F_E4M3,
                                            k, k * n, 0.0, dC, N.GRX_R_16BF, m, m * n, batch) == N.SUCCESS
        torch.cuda.synchronize()
        assert blas.execution_status() == N.SUCCESS
        return dC.float().cpu().numpy()

    Ad = oracle.decode("e4m3", Aq).reshape(batch, m, k)
    Bd = oracle.decode("e4m3", Bq).reshape(batch, n, k)
    narrow, wide = both(call, monkeypatch)
    assert np.array_equal(narrow, wide)
    for res in (narrow, wide):
        for b in range(batch):
            want = (Ad[b].astype(np.float64) @ Bd[b].T.astype(np.float64)) * sa[b][:, None] * sb[b][None, :]
            got = res[b * n * m:(b + 1) * n * m].reshape(n, m).T
            bad = np.abs(got - want) > TOL_ABS + TOL_REL * np.abs(want)
            assert not bad.any(), int(bad.sum())


CHILD = r"""
import sys; sys.path.insert(0, %r)
import torch
from grxcp_b200 import blas as B, _native as N
a = torch.randint(-128, 128, (512 * 512,), dtype=torch.int8, device="cuda")
c = torch.empty(512 * 512, dtype=torch.int32, device="cuda")
with B.Handle() as h:
    assert h.gemm_ex(0, 0, 512, 512, 512, 1.0, a, N.GRX_R_8I, 512, a, N.GRX_R_8I, 512, 0.0, c, N.GRX_R_32I, 512) == 0
    torch.cuda.synchronize()
    assert h.execution_status() == 0
""" % str(ROOT)


def _grids(**extra):
    env = dict(os.environ, GRX_PROFILE="1", **extra)
    r = subprocess.run([sys.executable, "-c", CHILD], env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    return [dict(f.split("=", 1) for f in l.split("|")[2:])["grid"] for l in r.stderr.splitlines()
            if l.startswith("GRXPROF|1|op=launch|") and "kernel=tc_gemm_kernel" in l]


def test_int8_512_launches_64_narrow_tiles():
    """4 x 2 tiles of 128 x 256, or 4 x 16 of 128 x 32 (64 <= 148 SMs)."""
    assert _grids(GRX_GEMM_WIDE_TILES="1") == ["8.1.1"]
    assert _grids() == ["64.1.1"]
