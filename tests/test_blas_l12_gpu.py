"""GPU gates of level-1/2 grxBLAS and the sgemm cycle probe, through the C-ABI.

Cases, fills and the poison conventions are the reference's
(tests/libs/test_grxblas_l12.cpp:79-300): small-integer values so every
comparison is exact, -12345 poison in every gap and overhang (a stray write
shows), NaN in y when beta == 0 (a kernel that reads y shows)."""
import ctypes as C

import numpy as np
import pytest
import torch

import oracle
from grxcp_b200 import _native as N

pytestmark = pytest.mark.gpu
POISON = np.float32(-12345.0)


def vidx(i, n, inc):
    return i * inc if inc > 0 else (n - 1 - i) * (-inc)


def span(n, inc):
    return 0 if n <= 0 else (n - 1) * abs(inc) + 1


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda()


AXPY = [(37, 1, 1), (21, 2, 3), (19, -1, 1), (19, 1, -2), (1, 1, 1)]


@pytest.mark.parametrize("n,incx,incy", AXPY)
def test_saxpy(blas, n, incx, incy):
    x = np.full(span(n, incx), POISON, np.float32)
    y = np.full(span(n, incy) + 8, POISON, np.float32)
    for i in range(n):
        x[vidx(i, n, incx)] = i + 1
        y[vidx(i, n, incy)] = 100 + i
    want = oracle.saxpy(n, 3.0, x, incx, y, incy)
    dx, dy = dev(x), dev(y)
    assert blas.saxpy(n, 3.0, dx, incx, dy, incy) == N.SUCCESS
    torch.cuda.synchronize()
    assert np.array_equal(dy.cpu().numpy(), want)


@pytest.mark.parametrize("n,incx,alpha", [(33, 1, 0.5), (17, 3, 2.0), (25, 1, 0.0)])
def test_sscal(blas, n, incx, alpha):
    x = np.full(span(n, incx) + 8, POISON, np.float32)
    for i in range(n):
        x[vidx(i, n, incx)] = i + 1
    want = oracle.sscal(n, alpha, x, incx)
    dx = dev(x)
    assert blas.sscal(n, alpha, dx, incx) == N.SUCCESS
    torch.cuda.synchronize()
    assert np.array_equal(dx.cpu().numpy(), want)


GEMV = [
    (0, 13, 7, 13, 1, 1, 2.0, 3.0), (0, 13, 7, 19, 1, 1, 2.0, 3.0), (0, 13, 7, 19, 2, 3, 2.0, 3.0),
    (0, 13, 7, 19, 1, 1, 1.0, 0.0), (0, 1, 9, 1, 1, 1, 2.0, 3.0), (0, 9, 1, 9, 1, 1, 2.0, 3.0),
    (1, 13, 7, 13, 1, 1, 2.0, 3.0), (1, 13, 7, 19, 1, 1, 2.0, 3.0), (1, 13, 7, 19, 2, -3, 2.0, 3.0),
    (1, 13, 7, 19, 1, 1, 1.0, 0.0), (1, 37, 5, 37, 1, 1, 2.0, 3.0),
    (0, 4000, 300, 4001, 1, 1, 2.0, 3.0), (1, 4000, 300, 4001, 1, -1, 2.0, 0.0),
]


@pytest.mark.parametrize("case", GEMV)
def test_sgemv(blas, case):
    tr, m, n, lda, incx, incy, alpha, beta = case
    rows, depth = (n, m) if tr else (m, n)
    A = np.full(lda * n, POISON, np.float32)
    for c in range(n):
        for r in range(m):
            A[r + c * lda] = ((r * 7 + c * 3) % 17) - 8
    x = np.full(span(depth, incx), POISON, np.float32)
    for i in range(depth):
        x[vidx(i, depth, incx)] = (i % 9) - 4
    y = np.full(span(rows, incy) + 8, POISON, np.float32)
    for i in range(rows):
        y[vidx(i, rows, incy)] = i + 1
    want = oracle.sgemv(tr, m, n, alpha, A, lda, x, incx, beta, y, incy)
    if beta == 0.0:
        for i in range(rows):
            y[vidx(i, rows, incy)] = np.nan
    dA, dx, dy = dev(A), dev(x), dev(y)
    assert blas.sgemv(tr, m, n, alpha, dA, lda, dx, incx, beta, dy, incy) == N.SUCCESS
    torch.cuda.synchronize()
    assert np.array_equal(dy.cpu().numpy(), want)
    assert np.array_equal(dA.cpu().numpy(), A), "sgemv leaves A alone"


def test_sgemm_cycle_probe(blas):
    """grxblasSetCycleProbe: the next sgemm writes one slot per CTA (reference
    include/grx/grxblas.h:229-242); too small a capacity is refused."""
    m = n = k = 300
    need = N.lib.grxblasCycleSlotsNeeded(None, m, n)
    # 300 x 300 fills no SM-count grid at 128 or 64, so sgemm runs 32 x 32 tiles: 10 x 10 CTAs.
    assert need == 100
    slots = torch.zeros(need * 3, dtype=torch.int64, device="cuda")  # 24-byte slots
    a = torch.ones(m * k, device="cuda")
    c = torch.zeros(m * n, device="cuda")
    assert blas.set_cycle_probe(slots, need - 1) == N.SUCCESS
    assert blas.sgemm(0, 0, m, n, k, 1.0, a, m, a, k, 0.0, c, m) == N.INVALID_VALUE
    assert blas.set_cycle_probe(slots, need) == N.SUCCESS
    assert blas.sgemm(0, 0, m, n, k, 1.0, a, m, a, k, 0.0, c, m) == N.SUCCESS
    torch.cuda.synchronize()
    raw = slots.cpu().numpy().view(np.uint64).reshape(need, 3)
    start, end = raw[:, 0], raw[:, 1]
    ids = (raw[:, 2] >> np.uint64(32)).astype(np.int64)
    assert np.all(end > start) and np.all(start > 0)
    assert sorted(ids.tolist()) == list(range(need))
    assert torch.all(c == k)
    assert blas.set_cycle_probe(None, 0) == N.SUCCESS
