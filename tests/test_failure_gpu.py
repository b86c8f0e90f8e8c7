"""Failure detection on the GPU without faulting it.

Every wait in the kernels is bounded. Here one CTA waits on an mbarrier that
nothing ever arrives at, through the same bounded-wait routine the GEMM and
attention kernels use; it must give up after the limit, report a timeout code
in the device error word, and leave the context usable (a GEMM right after it
still succeeds)."""
import time

import numpy as np
import pytest
import torch

from grxcp_b200 import _native as N

pytestmark = pytest.mark.gpu


def test_bounded_wait_times_out_and_context_survives(blas):
    t0 = time.time()
    code = N.lib.grxcpTestBoundedWait(50_000_000)  # 50 ms
    dt = time.time() - t0
    assert code == 5, f"expected the timeout code, got {code}"
    assert dt < 10
    # the context is intact: a GEMM still runs and is right
    a = torch.ones(64 * 64, device="cuda")
    c = torch.zeros(64 * 64, device="cuda")
    assert blas.sgemm(0, 0, 64, 64, 64, 1.0, a, 64, a, 64, 0.0, c, 64) == N.SUCCESS
    torch.cuda.synchronize()
    assert np.all(c.cpu().numpy() == 64.0)
    assert blas.execution_status() == N.SUCCESS
