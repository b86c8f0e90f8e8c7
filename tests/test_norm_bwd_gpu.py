"""GPU parity of grxdnnRMSNormBackward / grxdnnLayerNormBackward against the
fp64 oracle, through the C-ABI.

dx: |got - ref| <= 1e-2 + 2e-2*|ref| for 16-bit types (the grxDNN tolerance),
1e-4 + 1e-4*|ref| for fp32. dgamma / dbeta are fp32 sums over rows; each
column is held to 1e-3 of the sum of the absolute values of its terms (an
accumulation-error bound, since single terms are exact to fp32 rounding).
Covered: both dense-path widths, the scalar fallback (hidden not a multiple of
8, unaligned pitch), saved and recomputed statistics, repeat calls bit-equal,
rows == 0 zeroing the parameter gradients, and argument errors."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from grxcp_b200 import _native as N
from grxcp_b200 import dnn as D

pytestmark = pytest.mark.gpu

TORCH = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}


@pytest.fixture(scope="module")
def dh():
    h = D.Handle()
    yield h
    h.close()


def _inputs(rows, hidden, dt, seed, pitch=None):
    g = torch.Generator().manual_seed(seed)
    pitch = pitch or hidden
    xs = torch.randn(rows, pitch, generator=g).to(TORCH[dt])
    ds = torch.randn(rows, pitch, generator=g).to(TORCH[dt])
    gamma = (1 + 0.1 * torch.randn(hidden, generator=g)).float()
    beta = (0.1 * torch.randn(hidden, generator=g)).float()
    return xs, ds, gamma, beta


def _check(ln, dt, xs, ds, gamma, dx, dgamma, dbeta, hidden):
    x = xs[:, :hidden].float().numpy()
    dy = ds[:, :hidden].float().numpy()
    rdx, rdg, rdb = oracle.norm_bwd(ln, x, dy, gamma.numpy(), 1e-5)
    got = dx[:, :hidden].float().cpu().numpy()
    a, r = (1e-2, 2e-2) if dt != "f32" else (1e-4, 1e-4)
    bad = np.abs(got - rdx) > a + r * np.abs(rdx)
    assert not bad.any(), f"dx: {bad.sum()} out of tolerance, max err {np.abs(got - rdx).max()}"
    mu = x.mean(1, keepdims=True) if ln else 0.0
    var = ((x - mu) ** 2).mean(1, keepdims=True) if ln else (x.astype(np.float64) ** 2).mean(1, keepdims=True)
    xh = (x - mu) / np.sqrt(var + 1e-5)
    if dgamma is not None:
        bound = 1e-3 * np.abs(dy * xh).sum(0) + 1e-5
        err = np.abs(dgamma.cpu().numpy() - rdg)
        assert (err <= bound).all(), f"dgamma max err {err.max()}"
    if dbeta is not None:
        bound = 1e-3 * np.abs(dy).sum(0) + 1e-5
        err = np.abs(dbeta.cpu().numpy() - rdb)
        assert (err <= bound).all(), f"dbeta max err {err.max()}"


@pytest.mark.parametrize("dt", ["bf16", "f16", "f32"])
@pytest.mark.parametrize("ln", [False, True])
@pytest.mark.parametrize("rows,hidden", [(512, 4096), (300, 8192), (1000, 768)])
@pytest.mark.parametrize("saved", [True, False])
def test_norm_backward_dense(dh, dt, ln, rows, hidden, saved):
    if dt == "f32" and hidden > 4096:
        hidden = 4096  # widest fp32 row of the dense path; wider rows take the scalar path below
    xs, ds, gamma, beta = _inputs(rows, hidden, dt, 7 + hidden)
    x, dy, gm, bt = xs.cuda(), ds.cuda(), gamma.cuda(), beta.cuda()
    mean = torch.empty(rows, device="cuda") if ln else None
    rstd = torch.empty(rows, device="cuda")
    y = torch.empty_like(x)
    if saved:
        st = dh.layernorm(x, gm, bt, 1e-5, y, mean, rstd) if ln else dh.rmsnorm(x, gm, 1e-5, y, rstd)
        assert st == N.SUCCESS
    dx = torch.full_like(x, float("nan"))
    dg = torch.full((hidden,), float("nan"), device="cuda")
    db = torch.full((hidden,), float("nan"), device="cuda") if ln else None
    for rep in range(2):
        if ln:
            st = dh.layernorm_backward(dy, x, gm, 1e-5, dx, mean if saved else None, rstd if saved else None, dg, db)
        else:
            st = dh.rmsnorm_backward(dy, x, gm, 1e-5, dx, rstd if saved else None, dg)
        assert st == N.SUCCESS
        torch.cuda.synchronize()
        assert dh.execution_status() == N.SUCCESS
        if rep == 0:
            first = (dx.clone(), dg.clone(), None if db is None else db.clone())
    assert torch.equal(first[0], dx) and torch.equal(first[1], dg), "repeat call differs"
    if ln:
        assert torch.equal(first[2], db)
    _check(ln, dt, xs, ds, gamma, dx.cpu(), dg, db, hidden)


@pytest.mark.parametrize("ln", [False, True])
@pytest.mark.parametrize("hidden,pitch", [(1000, 1003), (4100, 4100), (12288, 12288)])
def test_norm_backward_scalar_path(dh, ln, hidden, pitch):
    """Rows that defeat the 16-byte dense path: odd width or pitch, or wider
    than 8192 bf16 elements. Statistics recomputed (no saved ones)."""
    rows = 96
    xs, ds, gamma, _ = _inputs(rows, hidden, "bf16", 3, pitch)
    x, dy, gm = xs.cuda(), ds.cuda(), gamma.cuda()
    dx = torch.zeros_like(x)
    dg = torch.full((hidden,), float("nan"), device="cuda")
    db = torch.full((hidden,), float("nan"), device="cuda") if ln else None
    lib = N.lib
    if ln:
        st = lib.grxdnnLayerNormBackward(dh.h, rows, hidden, dy.data_ptr(), N.GRX_R_16BF, pitch, x.data_ptr(),
                                         N.GRX_R_16BF, pitch, gm.data_ptr(), None, None, 1e-5, dx.data_ptr(),
                                         N.GRX_R_16BF, pitch, dg.data_ptr(), db.data_ptr())
    else:
        st = lib.grxdnnRMSNormBackward(dh.h, rows, hidden, dy.data_ptr(), N.GRX_R_16BF, pitch, x.data_ptr(),
                                       N.GRX_R_16BF, pitch, gm.data_ptr(), None, 1e-5, dx.data_ptr(), N.GRX_R_16BF,
                                       pitch, dg.data_ptr())
    assert st == N.SUCCESS
    torch.cuda.synchronize()
    assert dh.execution_status() == N.SUCCESS
    _check(ln, "bf16", xs, ds, gamma, dx.cpu(), dg, db, hidden)
    if pitch > hidden:
        assert torch.equal(dx[:, hidden:].cpu(), torch.zeros(rows, pitch - hidden, dtype=torch.bfloat16)), \
            "pitch padding of dx was written"


def test_norm_backward_empty_and_errors(dh):
    lib = N.lib
    dg = torch.full((64,), 5.0, device="cuda")
    db = torch.full((64,), 5.0, device="cuda")
    one = torch.zeros(64 * 8, device="cuda", dtype=torch.bfloat16)
    g = torch.ones(64, device="cuda")
    # rows == 0: parameter gradients are sums over nothing
    assert lib.grxdnnLayerNormBackward(dh.h, 0, 64, None, N.GRX_R_16BF, 64, None, N.GRX_R_16BF, 64, g.data_ptr(),
                                       None, None, 1e-5, None, N.GRX_R_16BF, 64, dg.data_ptr(),
                                       db.data_ptr()) == N.SUCCESS
    torch.cuda.synchronize()
    assert (dg == 0).all() and (db == 0).all()
    p = one.data_ptr()
    # mean without rstd
    mean = torch.zeros(8, device="cuda")
    assert lib.grxdnnLayerNormBackward(dh.h, 8, 64, p, N.GRX_R_16BF, 64, p, N.GRX_R_16BF, 64, g.data_ptr(),
                                       mean.data_ptr(), None, 1e-5, p, N.GRX_R_16BF, 64, None,
                                       None) == N.INVALID_VALUE
    # dy of another type
    assert lib.grxdnnRMSNormBackward(dh.h, 8, 64, p, N.GRX_R_16F, 64, p, N.GRX_R_16BF, 64, g.data_ptr(), None, 1e-5,
                                     p, N.GRX_R_16BF, 64, None) == N.NOT_SUPPORTED
    # pitch below width, null dy, null handle
    assert lib.grxdnnRMSNormBackward(dh.h, 8, 64, p, N.GRX_R_16BF, 63, p, N.GRX_R_16BF, 64, g.data_ptr(), None, 1e-5,
                                     p, N.GRX_R_16BF, 64, None) == N.INVALID_VALUE
    assert lib.grxdnnRMSNormBackward(dh.h, 8, 64, None, N.GRX_R_16BF, 64, p, N.GRX_R_16BF, 64, g.data_ptr(), None,
                                     1e-5, p, N.GRX_R_16BF, 64, None) == N.INVALID_VALUE
    assert lib.grxdnnRMSNormBackward(None, 8, 64, p, N.GRX_R_16BF, 64, p, N.GRX_R_16BF, 64, g.data_ptr(), None,
                                     1e-5, p, N.GRX_R_16BF, 64, None) == N.NOT_INITIALIZED


@pytest.mark.parametrize("ln", [False, True])
def test_norm_backward_l2_prefetch_changes_no_bits(dh, ln, monkeypatch):
    """The dense kernels ask L2 for each CTA's next row (bulk prefetch); that
    moves no data the arithmetic sees, so dx, dgamma and dbeta equal the
    results with the prefetch off (GRX_NORM_BWD_NO_PREFETCH=1) bit for bit."""
    rows, hidden = 3000, 8192
    xs, ds, gamma, beta = _inputs(rows, hidden, "bf16", 21)
    x, dy, gm, bt = xs.cuda(), ds.cuda(), gamma.cuda(), beta.cuda()
    mean = torch.empty(rows, device="cuda")
    rstd = torch.empty(rows, device="cuda")
    y = torch.empty_like(x)
    assert (dh.layernorm(x, gm, bt, 1e-5, y, mean, rstd) if ln else dh.rmsnorm(x, gm, 1e-5, y, rstd)) == N.SUCCESS

    def run():
        dx = torch.full_like(x, float("nan"))
        dg = torch.full((hidden,), float("nan"), device="cuda")
        db = torch.full((hidden,), float("nan"), device="cuda")
        if ln:
            st = dh.layernorm_backward(dy, x, gm, 1e-5, dx, mean, rstd, dg, db)
        else:
            st = dh.rmsnorm_backward(dy, x, gm, 1e-5, dx, rstd, dg)
        assert st == N.SUCCESS
        torch.cuda.synchronize()
        assert dh.execution_status() == N.SUCCESS
        return dx, dg, db

    a = run()
    monkeypatch.setenv("GRX_NORM_BWD_NO_PREFETCH", "1")
    b = run()
    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])
    if ln:
        assert torch.equal(a[2], b[2])
    _check(ln, "bf16", xs, ds, gamma, a[0].cpu(), a[1], a[2] if ln else None, hidden)
