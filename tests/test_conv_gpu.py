"""GPU parity of grxdnnConv2dForward and grxdnnPooling2dForward against the
fp64 oracle, through the C-ABI.

conv2d: bf16 inputs with a channel count that is a multiple of 64 run the
tcgen05 implicit GEMM (4-D TMA loads of strided pixel blocks, padding from the
loads' out-of-range fill); the rest run the direct kernel. Tolerance
|got - ref| <= 1e-2 + 2e-2 |ref| (the grxDNN bound). Covered: 1x1, 3x3 with
padding, stride 2, dilation, output widths that do not fill a pixel block,
output channels that do not fill a 128-row tile, bias + activation, beta,
fp32 output, the direct path (3 input channels, fp32 tensors), and argument
errors. Pooling: max (exact), both averages, with padding and strides."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from grxcp_b200 import _native as N
from grxcp_b200 import dnn as D

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dh():
    h = D.Handle()
    yield h
    h.close()


def _close(got, ref):
    got = np.asarray(got, np.float64)
    bad = np.abs(got - ref) > 1e-2 + 2e-2 * np.abs(ref)
    return not bad.any(), int(bad.sum()), float(np.abs(got - ref).max())


def _conv_case(dh, n, h, w, c, k, r, s, pad, stride, dil, dt=torch.bfloat16, out=torch.bfloat16, bias=False,
               act=0, beta=None, seed=0):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(n, h, w, c, generator=g).to(dt)
    f = (torch.randn(k, r, s, c, generator=g) / (r * s * c) ** 0.5).to(dt)
    b = (torch.randn(k, generator=g) * 0.5) if bias else None
    ref = oracle.conv2d(x.float().numpy(), f.float().numpy(), pad, stride, dil)
    y0 = torch.randn(ref.shape, generator=g).to(out)
    if beta is not None:
        ref = ref + beta * y0.double().numpy()
    if bias:
        ref = ref + b.double().numpy()
    if act == N.ACT_RELU:
        ref = np.maximum(ref, 0)
    elif act == N.ACT_GELU_TANH:
        ref = oracle.gelu(ref.astype(np.float32), 1)
    y = y0.cuda() if beta is not None else torch.full(ref.shape, float("nan"), dtype=out, device="cuda")
    st = dh.conv2d(x.cuda(), f.cuda(), y, pad, stride, dil, None if b is None else b.cuda(), act,
                   beta=beta if beta is not None else None)
    assert st == N.SUCCESS, N.STATUS.get(st, st)
    torch.cuda.synchronize()
    assert dh.execution_status() == N.SUCCESS
    ok, nbad, mx = _close(y.float().cpu().numpy(), ref)
    assert ok, f"{nbad} of {ref.size} out of tolerance, max err {mx}"


@pytest.mark.parametrize("n,h,w,c,k,r,s,pad,stride,dil", [
    (2, 14, 14, 64, 128, 3, 3, (1, 1), (1, 1), (1, 1)),    # 3x3 same, 16x16 pixel blocks
    (2, 28, 28, 128, 256, 1, 1, (0, 0), (1, 1), (1, 1)),   # 1x1, 32-wide blocks
    (2, 56, 56, 64, 64, 3, 3, (1, 1), (2, 2), (1, 1)),     # stride 2
    (1, 32, 40, 64, 64, 5, 5, (2, 2), (1, 1), (2, 2)),     # dilation 2, ragged blocks
    (3, 7, 7, 192, 96, 3, 3, (1, 1), (1, 1), (1, 1)),      # 7-wide output, 96 channels (partial M tile)
    (1, 9, 300, 64, 128, 1, 3, (0, 1), (1, 2), (1, 1)),    # wide rows, stride 2 along w only
])
def test_conv2d_tensor_path(dh, n, h, w, c, k, r, s, pad, stride, dil):
    _conv_case(dh, n, h, w, c, k, r, s, pad, stride, dil, seed=h * w + k)


def test_conv2d_bias_relu_fp32_out(dh):
    _conv_case(dh, 2, 16, 16, 64, 128, 3, 3, (1, 1), (1, 1), (1, 1), out=torch.float32, bias=True,
               act=N.ACT_RELU, seed=5)


def test_conv2d_bias_gelu_beta(dh):
    _conv_case(dh, 1, 12, 12, 128, 64, 3, 3, (1, 1), (1, 1), (1, 1), bias=True, act=N.ACT_GELU_TANH,
               beta=0.5, out=torch.float32, seed=6)


def test_conv2d_direct_first_layer(dh):
    """3 input channels (a stem conv) cannot be tiled by 64-channel boxes: direct kernel."""
    _conv_case(dh, 2, 32, 32, 3, 64, 7, 7, (3, 3), (2, 2), (1, 1), seed=7)


def test_conv2d_direct_fp32(dh):
    _conv_case(dh, 1, 10, 11, 16, 24, 3, 3, (1, 1), (1, 1), (1, 1), dt=torch.float32, out=torch.float32, bias=True,
               seed=8)


def test_conv2d_errors(dh):
    x = torch.zeros(1, 8, 8, 64, dtype=torch.bfloat16, device="cuda")
    w = torch.zeros(64, 3, 3, 64, dtype=torch.bfloat16, device="cuda")
    y = torch.zeros(1, 6, 6, 64, dtype=torch.bfloat16, device="cuda")
    assert dh.conv2d(x, w, y, stride=(0, 1)) == N.INVALID_VALUE
    assert dh.conv2d(x, w, y, activation=9) == N.INVALID_VALUE
    big = torch.zeros(64, 11, 11, 64, dtype=torch.bfloat16, device="cuda")  # filter larger than the padded image
    assert dh.conv2d(x, big, y) == N.INVALID_VALUE
    wh = torch.zeros(64, 3, 3, 64, dtype=torch.float16, device="cuda")
    assert dh.conv2d(x, wh, y) == N.NOT_SUPPORTED  # mixed types


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("mode", [0, 1, 2])
@pytest.mark.parametrize("window,pad,stride", [((3, 3), (1, 1), (2, 2)), ((2, 2), (0, 0), (2, 2)),
                                               ((3, 2), (1, 0), (1, 2)), ((4, 3), (1, 1), (2, 2))])
@pytest.mark.parametrize("c", [40, 36])  # 16-bit: 8-channel vector kernel / element kernel
def test_pool2d(dh, dt, mode, window, pad, stride, c):
    g = torch.Generator().manual_seed(11)
    x = torch.randn(2, 15, 17, c, generator=g).to(dt)
    ref = oracle.pool2d(x.double().numpy(), window, pad, stride, mode)
    y = torch.full(ref.shape, float("nan"), dtype=dt, device="cuda")
    assert dh.pool2d(x.cuda(), y, window, pad, stride, mode) == N.SUCCESS
    torch.cuda.synchronize()
    got = y.double().cpu().numpy()
    if mode == 0:
        assert np.array_equal(got, ref), "max pooling must be exact"
    else:
        tol = 1e-2 if dt == torch.bfloat16 else 1e-5
        assert np.allclose(got, ref, rtol=tol, atol=tol)


CHILD = r"""
import sys; sys.path.insert(0, %r)
import torch
from grxcp_b200 import dnn as D
h = D.Handle()
for (hw, c, k, r) in [(14, 64, 128, 3), (7, 192, 96, 3)]:
    x = torch.randn(2, hw, hw, c, device="cuda").to(torch.bfloat16)
    w = torch.randn(k, r, r, c, device="cuda").to(torch.bfloat16)
    y = torch.empty(2, hw, hw, k, device="cuda").to(torch.bfloat16)
    assert h.conv2d(x, w, y, pad=(1, 1)) == 0
torch.cuda.synchronize()
"""


def test_conv2d_runs_on_tensor_cores():
    """The 64-channel-multiple shapes above must take the tcgen05 kernel, not the direct fallback."""
    import os
    import subprocess
    import sys
    from pathlib import Path

    root = Path(__file__).resolve().parent.parent
    env = dict(os.environ, GRX_PROFILE="1")
    r = subprocess.run([sys.executable, "-c", CHILD % str(root)], env=env, capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    names = [l.split("kernel=")[1].split("|")[0] for l in r.stderr.splitlines() if "op=launch" in l]
    assert names == ["tc_gemm_kernel", "tc_gemm_kernel"], names
