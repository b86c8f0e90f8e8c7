"""GPU parity of grxDNN (RMSNorm, LayerNorm, attention forward) against the
fp64 oracle, through the C-ABI. Tolerance |got - ref| <= 1e-2 + 2e-2*|ref|
(bf16 outputs); fp32 statistics within 1e-4 relative."""
from __future__ import annotations

import math

import numpy as np
import pytest
import torch

import oracle
from grxcp_b200 import _native as N

pytestmark = pytest.mark.gpu

TOL_ABS, TOL_REL = 1e-2, 2e-2


def close(got, ref, abs_tol=TOL_ABS, rel_tol=TOL_REL):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    bad = ~(np.abs(got - ref) <= abs_tol + rel_tol * np.abs(ref))
    return not bad.any(), int(bad.sum())


def _norm_inputs(rows, hidden, dtype, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(rows, hidden, device="cuda", generator=g).to(dtype)
    gamma = 1 + 0.02 * torch.randn(hidden, device="cuda", generator=g)
    beta = 0.02 * torch.randn(hidden, device="cuda", generator=g)
    return x, gamma, beta


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("rows,hidden", [(64, 8192), (37, 1000), (5, 4096), (300, 128), (3, 24576)])
def test_rmsnorm(dnn, dtype, rows, hidden):
    x, gamma, _ = _norm_inputs(rows, hidden, dtype)
    y = torch.full_like(x, float("nan"))
    rstd = torch.empty(rows, device="cuda")
    assert dnn.rmsnorm(x, gamma, 1e-5, y, rstd) == N.SUCCESS
    torch.cuda.synchronize()
    ref, ref_rstd = oracle.rmsnorm(x.float().cpu().numpy(), gamma.cpu().numpy(), 1e-5)
    ok, nbad = close(y.float().cpu().numpy(), ref)
    assert ok, nbad
    assert np.allclose(rstd.cpu().numpy(), ref_rstd, rtol=1e-4)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("rows,hidden", [(64, 8192), (37, 1000), (300, 128), (3, 24576)])
def test_layernorm(dnn, dtype, rows, hidden):
    x, gamma, beta = _norm_inputs(rows, hidden, dtype, 1)
    y = torch.full_like(x, float("nan"))
    mean = torch.empty(rows, device="cuda")
    rstd = torch.empty(rows, device="cuda")
    assert dnn.layernorm(x, gamma, beta, 1e-5, y, mean, rstd) == N.SUCCESS
    torch.cuda.synchronize()
    ref, rm, rr = oracle.layernorm(x.float().cpu().numpy(), gamma.cpu().numpy(), beta.cpu().numpy(), 1e-5)
    ok, nbad = close(y.float().cpu().numpy(), ref)
    assert ok, nbad
    assert np.allclose(mean.cpu().numpy(), rm, atol=1e-5)
    assert np.allclose(rstd.cpu().numpy(), rr, rtol=1e-4)


def test_norm_strided_rows_and_unaligned(dnn):
    """Row pitch larger than hidden, and a pitch that defeats 16-byte vectors."""
    base = torch.randn(20, 1031, device="cuda").to(torch.bfloat16)
    x = base[:, 3:1003]  # pitch 1031, offset 3 elements: unaligned
    gamma = torch.ones(1000, device="cuda") * 1.1
    y = torch.full((20, 1040), float("nan"), device="cuda", dtype=torch.bfloat16)
    yv = y[:, :1000]
    assert dnn.rmsnorm(x, gamma, 1e-5, yv, None, ldx=1031, ldy=1040) == N.SUCCESS
    torch.cuda.synchronize()
    ref, _ = oracle.rmsnorm(x.float().cpu().numpy(), gamma.cpu().numpy(), 1e-5)
    ok, nbad = close(yv.float().cpu().numpy(), ref)
    assert ok, nbad
    assert torch.isnan(y[:, 1000:].float()).all(), "pitch padding written"


def test_norm_config3_full(dnn):
    """BASELINE config 3 at full size [65536, 8192] bf16: full comparison of LayerNorm and
    RMSNorm outputs against the oracle for 512 sampled rows, plus every row's statistics."""
    rows, hidden = 65536, 8192
    x, gamma, beta = _norm_inputs(rows, hidden, torch.bfloat16, 3)
    y = torch.empty_like(x)
    mean = torch.empty(rows, device="cuda")
    rstd = torch.empty(rows, device="cuda")
    assert dnn.layernorm(x, gamma, beta, 1e-5, y, mean, rstd) == N.SUCCESS
    torch.cuda.synchronize()
    sel = torch.as_tensor(np.random.default_rng(0).choice(rows, 512, replace=False), device="cuda")
    ref, rm, rr = oracle.layernorm(x[sel].float().cpu().numpy(), gamma.cpu().numpy(), beta.cpu().numpy(), 1e-5)
    ok, nbad = close(y[sel].float().cpu().numpy(), ref)
    assert ok, nbad
    xs = x.float()
    mu = xs.mean(1)
    assert torch.allclose(mean, mu, atol=1e-4)
    assert torch.allclose(rstd, 1 / torch.sqrt(xs.var(1, unbiased=False) + 1e-5), rtol=1e-3)
    assert dnn.rmsnorm(x, gamma, 1e-5, y, rstd) == N.SUCCESS
    torch.cuda.synchronize()
    ref, _ = oracle.rmsnorm(x[sel].float().cpu().numpy(), gamma.cpu().numpy(), 1e-5)
    ok, nbad = close(y[sel].float().cpu().numpy(), ref)
    assert ok, nbad


# ------------------------------------------------------------------ attention

def _attn(dnn, B, H, S, causal, seed=0, Sk=None):
    Sk = S if Sk is None else Sk
    g = torch.Generator(device="cuda").manual_seed(seed)
    q = torch.randn(B, H, S, 128, device="cuda", generator=g).to(torch.bfloat16)
    k = torch.randn(B, H, Sk, 128, device="cuda", generator=g).to(torch.bfloat16)
    v = torch.randn(B, H, Sk, 128, device="cuda", generator=g).to(torch.bfloat16)
    o = torch.full_like(q, float("nan"))
    lse = torch.full((B, H, S), float("nan"), device="cuda")
    scale = 1 / math.sqrt(128)
    st = dnn.attention(q, k, v, o, scale, causal, lse)
    assert st == N.SUCCESS, N.STATUS[st]
    torch.cuda.synchronize()
    assert dnn.execution_status() == N.SUCCESS
    return q, k, v, o, lse, scale


@pytest.mark.parametrize("causal", [True, False])
@pytest.mark.parametrize("B,H,S", [(1, 2, 128), (2, 3, 384), (1, 2, 200), (1, 1, 1), (2, 2, 700)])
def test_attention_small(dnn, B, H, S, causal):
    q, k, v, o, lse, scale = _attn(dnn, B, H, S, causal, seed=S)
    ro, rl = oracle.attention(q.float().reshape(B * H, S, 128).cpu().numpy(),
                              k.float().reshape(B * H, S, 128).cpu().numpy(),
                              v.float().reshape(B * H, S, 128).cpu().numpy(), scale, causal)
    ok, nbad = close(o.float().reshape(B * H, S, 128).cpu().numpy(), ro)
    assert ok, nbad
    assert np.allclose(lse.reshape(B * H, S).cpu().numpy(), rl, atol=2e-3, rtol=1e-3)


def test_attention_noncausal_longer_keys(dnn):
    B, H, S, Sk = 1, 2, 256, 640
    q, k, v, o, lse, scale = _attn(dnn, B, H, S, False, seed=4, Sk=Sk)
    ro, rl = oracle.attention(q.float().reshape(B * H, S, 128).cpu().numpy(),
                              k.float().reshape(B * H, Sk, 128).cpu().numpy(),
                              v.float().reshape(B * H, Sk, 128).cpu().numpy(), scale, False)
    ok, nbad = close(o.float().reshape(B * H, S, 128).cpu().numpy(), ro)
    assert ok, nbad


def test_attention_config4_sampled(dnn):
    """BASELINE config 4 at full size (B=8, H=32, S=4096, causal): sampled (b, h) pairs,
    query rows at the start, the tile seams and the end, full O rows and LSE."""
    B, H, S = 8, 32, 4096
    q, k, v, o, lse, scale = _attn(dnn, B, H, S, True, seed=1)
    pairs = np.array([0, 37, 129, 255])
    rows = np.unique(np.concatenate([np.arange(0, 4), [127, 128, 129, 2047, 2048], np.arange(S - 4, S)]))
    qf = q.reshape(B * H, S, 128)[torch.as_tensor(pairs, device="cuda")].float().cpu().numpy()
    kf = k.reshape(B * H, S, 128)[torch.as_tensor(pairs, device="cuda")].float().cpu().numpy()
    vf = v.reshape(B * H, S, 128)[torch.as_tensor(pairs, device="cuda")].float().cpu().numpy()
    go = o.reshape(B * H, S, 128)[torch.as_tensor(pairs, device="cuda")].float().cpu().numpy()
    gl = lse.reshape(B * H, S)[torch.as_tensor(pairs, device="cuda")].cpu().numpy()
    for r in rows:
        ro, rl = oracle.attention(qf, kf, vf, scale, True, q0=int(r), q1=int(r) + 1)
        ok, nbad = close(go[:, r, :], ro[:, 0, :])
        assert ok, (r, nbad)
        assert np.allclose(gl[:, r], rl[:, 0], atol=2e-3, rtol=1e-3)
    assert not torch.isnan(o.float()).any()


def test_attention_refusals(dnn):
    from grxcp_b200.dnn import attn_desc

    q = torch.zeros(1, 1, 128, 64, dtype=torch.bfloat16, device="cuda")
    d = attn_desc(q)
    assert dnn.attention(q, q, q, q, 0.1, True, descs=(d, d, d, d)) == N.NOT_SUPPORTED  # head_dim 64
    q2 = torch.zeros(1, 1, 128, 128, dtype=torch.float16, device="cuda")
    assert dnn.attention(q2, q2, q2, q2, 0.1, True) == N.NOT_SUPPORTED  # fp16


# ------------------------------------------------------------------ softmax / GELU

@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("rows,cols", [(64, 4096), (33, 1000), (5, 32768), (300, 7)])
def test_softmax(dnn, dtype, rows, cols):
    g = torch.Generator(device="cuda").manual_seed(rows + cols)
    x = (torch.randn(rows, cols, device="cuda", generator=g) * 3).to(dtype)
    y = torch.full_like(x, float("nan"))
    assert dnn.softmax(x, y) == N.SUCCESS
    torch.cuda.synchronize()
    ref = oracle.softmax(x.float().cpu().numpy())
    tol = (1e-5, 1e-4) if dtype == torch.float32 else (TOL_ABS, TOL_REL)
    ok, nbad = close(y.float().cpu().numpy(), ref, *tol)
    assert ok, nbad
    assert np.allclose(y.float().sum(1).cpu().numpy(), 1.0, atol=5e-3 if dtype != torch.float32 else 1e-5)


def test_softmax_strided_and_refusals(dnn):
    base = torch.randn(10, 517, device="cuda").to(torch.bfloat16)
    x = base[:, 1:501]
    y = torch.zeros(10, 512, device="cuda", dtype=torch.bfloat16)
    assert dnn.softmax(x, y[:, :500], ldx=517, ldy=512) == N.SUCCESS
    torch.cuda.synchronize()
    ok, nbad = close(y[:, :500].float().cpu().numpy(), oracle.softmax(x.float().cpu().numpy()))
    assert ok, nbad
    assert torch.all(y[:, 500:] == 0)
    z = torch.zeros(4, 8, device="cuda", dtype=torch.int8)
    assert dnn.softmax(z, z) == N.NOT_SUPPORTED


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_gelu_erf_16bit_whole_range(dnn, dtype):
    """16-bit erf-form GELU uses the Abramowitz & Stegun 7.1.26 erf (abs. error
    <= 1.5e-7). Every value on a dense grid over [-12, 12] plus the type's
    extremes is checked against the fp64 oracle: the far negative tail stays a
    small negative number (no cancellation to 0 or NaN) and large positive x
    returns x."""
    grid = torch.linspace(-12, 12, 1 << 16, device="cuda")
    big = torch.tensor([-60000.0, -1000.0, -40.0, 40.0, 1000.0, 60000.0], device="cuda")
    x = torch.cat([grid, big]).to(dtype)
    y = torch.empty_like(x)
    assert dnn.gelu(x, y, 0) == N.SUCCESS
    torch.cuda.synchronize()
    got = y.float().cpu().numpy()
    ref = oracle.gelu(x.float().cpu().numpy(), 0)
    assert np.all(np.isfinite(got))
    ok, nbad = close(got, ref, TOL_ABS, TOL_REL)
    assert ok, nbad
    xs = x.float().cpu().numpy()
    tail = (xs < -3) & (xs > -8) & (np.abs(ref) > torch.finfo(dtype).tiny)  # representable as a normal value
    # the tail keeps its sign and magnitude (A&S's relative error grows toward x = -8, where the
    # values are below 1e-14; measured within 4 % there)
    assert np.all(got[tail] < 0) and np.all(np.abs(got[tail] - ref[tail]) <= 6e-2 * np.abs(ref[tail]))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("mode", [0, 1])
@pytest.mark.parametrize("n", [1 << 20, 12345])
def test_gelu(dnn, dtype, mode, n):
    g = torch.Generator(device="cuda").manual_seed(n + mode)
    x = (torch.randn(n, device="cuda", generator=g) * 3).to(dtype)
    y = torch.empty_like(x)
    assert dnn.gelu(x, y, mode) == N.SUCCESS
    torch.cuda.synchronize()
    ref = oracle.gelu(x.float().cpu().numpy(), mode)
    tol = (1e-5, 1e-5) if dtype == torch.float32 else (TOL_ABS, TOL_REL)
    ok, nbad = close(y.float().cpu().numpy(), ref, *tol)
    assert ok, nbad
    # in place
    assert dnn.gelu(x, x, mode) == N.SUCCESS
    torch.cuda.synchronize()
    assert torch.equal(x, y)


# ------------------------------------------------------------------ softmax / GELU backward

@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("rows,cols", [(64, 4096), (33, 1000), (16, 8192), (5, 1003)])
def test_softmax_backward(dnn, dtype, rows, cols):
    """dx = y (dy - sum dy y) against the fp64 oracle, from the library's own forward output."""
    g = torch.Generator(device="cuda").manual_seed(rows + cols)
    x = (torch.randn(rows, cols, device="cuda", generator=g) * 3).to(dtype)
    dy = torch.randn(rows, cols, device="cuda", generator=g).to(dtype)
    y = torch.empty_like(x)
    dx = torch.full_like(x, float("nan"))
    assert dnn.softmax(x, y) == N.SUCCESS
    assert dnn.softmax_backward(y, dy, dx) == N.SUCCESS
    torch.cuda.synchronize()
    ref = oracle.softmax_bwd(y.double().cpu().numpy(), dy.double().cpu().numpy())
    got = dx.double().cpu().numpy()
    tol = 1e-2 if dtype == torch.bfloat16 else 1e-5
    assert np.all(np.abs(got - ref) <= tol * (1e-2 + np.abs(ref)) + 1e-6), np.abs(got - ref).max()
    # in place (dx aliasing dy, as training code does): the same bits as out of place
    dy2 = dy.clone()
    assert dnn.softmax_backward(y, dy2, dy2) == N.SUCCESS
    y2 = x.clone()
    assert dnn.softmax(y2, y2) == N.SUCCESS
    torch.cuda.synchronize()
    assert torch.equal(dy2, dx)
    assert torch.equal(y2, y)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("mode", [0, 1])
def test_gelu_backward(dnn, dtype, mode):
    g = torch.Generator(device="cuda").manual_seed(3 + mode)
    x = (torch.randn(100003, device="cuda", generator=g) * 3).to(dtype)
    dy = torch.randn(100003, device="cuda", generator=g).to(dtype)
    dx = torch.full_like(x, float("nan"))
    assert dnn.gelu_backward(x, dy, dx, mode) == N.SUCCESS
    torch.cuda.synchronize()
    ref = oracle.gelu_bwd(x.double().cpu().numpy(), dy.double().cpu().numpy(), mode)
    got = dx.double().cpu().numpy()
    a, r = (1e-2, 2e-2) if dtype == torch.bfloat16 else (1e-5, 1e-5)
    assert np.all(np.abs(got - ref) <= a + r * np.abs(ref)), np.abs(got - ref).max()
    # in place (dx aliasing dy): the same bits as out of place
    dy2 = dy.clone()
    assert dnn.gelu_backward(x, dy2, dy2, mode) == N.SUCCESS
    torch.cuda.synchronize()
    assert torch.equal(dy2, dx)
