"""Failure detection on a GPU, with no GPU fault.

* Host-side injection (GRX_FAULT_INJECT): a device allocation the library makes
  fails -> ALLOC_FAILED; kernel-path resolution fails -> NOT_INITIALIZED; the
  handle works again once the fault is gone.
* The real abort path of the tensor-core GEMM: a child process sets a 1 ms
  bounded-wait limit and runs one 128 x 256 tile with k = 2^20 (about 7 ms of
  MMAs), so the epilogue warps give up waiting for the accumulator. The kernel
  records the timeout, the MMA issuer drains its MMAs, the producer lets its
  TMA loads land, TMEM is freed and the kernel returns;
  grxblasGetExecutionStatus reports EXECUTION_FAILED and the next GemmEx in the
  same process is correct. Nothing waits without a limit."""
import os
import subprocess
import sys
import textwrap
from pathlib import Path

import pytest
import torch

from grxcp_b200 import _native as N
from grxcp_b200 import blas as B
from grxcp_b200 import dnn as D

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parent.parent


def _small(dev):
    g = torch.Generator(device="cuda").manual_seed(4)
    a = torch.randn(256 * 256, device=dev, generator=g).to(torch.bfloat16)
    return a, torch.empty(256 * 256, device=dev, dtype=torch.float32)


def test_alloc_failure_on_first_use(dev, monkeypatch):
    a, c = _small(dev)
    with B.Handle() as h:
        monkeypatch.setenv("GRX_FAULT_INJECT", "alloc")
        assert h.gemm_ex(0, 0, 256, 256, 256, 1.0, a, N.GRX_R_16BF, 256, a, N.GRX_R_16BF, 256, 0.0, c, N.GRX_R_32F,
                         256) == N.ALLOC_FAILED
        monkeypatch.delenv("GRX_FAULT_INJECT")
        assert h.gemm_ex(0, 0, 256, 256, 256, 1.0, a, N.GRX_R_16BF, 256, a, N.GRX_R_16BF, 256, 0.0, c, N.GRX_R_32F,
                         256) == N.SUCCESS
        torch.cuda.synchronize()
        assert h.execution_status() == N.SUCCESS
    x = torch.randn(4, 1024, device=dev).to(torch.bfloat16)
    y = torch.empty_like(x)
    gamma = torch.ones(1024, device=dev)
    with D.Handle() as dh:
        monkeypatch.setenv("GRX_FAULT_INJECT", "alloc")
        assert dh.rmsnorm(x, gamma, 1e-5, y) == N.ALLOC_FAILED
        monkeypatch.delenv("GRX_FAULT_INJECT")
        assert dh.rmsnorm(x, gamma, 1e-5, y) == N.SUCCESS


def test_workspace_alloc_failure(dev, monkeypatch):
    a, c = _small(dev)
    with B.Handle() as h:
        assert h.gemm_ex(0, 0, 256, 256, 256, 1.0, a, N.GRX_R_16BF, 256, a, N.GRX_R_16BF, 256, 0.0, c, N.GRX_R_32F,
                         256) == N.SUCCESS
        monkeypatch.setenv("GRX_FAULT_INJECT", "alloc")
        # lda = 255 is not 16-byte aligned: A must be packed into the handle's workspace
        assert h.gemm_ex(0, 0, 255, 256, 256, 1.0, a, N.GRX_R_16BF, 255, a, N.GRX_R_16BF, 256, 0.0, c, N.GRX_R_32F,
                         256) == N.ALLOC_FAILED
        # an aligned call needs no workspace and still runs
        assert h.gemm_ex(0, 0, 256, 256, 256, 1.0, a, N.GRX_R_16BF, 256, a, N.GRX_R_16BF, 256, 0.0, c, N.GRX_R_32F,
                         256) == N.SUCCESS
        torch.cuda.synchronize()
        assert h.execution_status() == N.SUCCESS


def test_module_resolution_failure(dev, monkeypatch):
    a, c = _small(dev)
    with B.Handle() as h:
        monkeypatch.setenv("GRX_FAULT_INJECT", "module")
        assert h.sgemm(0, 0, 16, 16, 16, 1.0, c, 16, c, 16, 0.0, c, 16) == N.NOT_INITIALIZED
        assert h.gemm_ex(0, 0, 256, 256, 256, 1.0, a, N.GRX_R_16BF, 256, a, N.GRX_R_16BF, 256, 0.0, c, N.GRX_R_32F,
                         256) == N.NOT_INITIALIZED
        monkeypatch.delenv("GRX_FAULT_INJECT")
        assert h.sgemm(0, 0, 16, 16, 16, 1.0, c, 16, c, 16, 0.0, c, 16) == N.SUCCESS
        torch.cuda.synchronize()


CHILD = textwrap.dedent("""
    import sys, torch
    sys.path.insert(0, sys.argv[1])
    from grxcp_b200 import _native as N
    from grxcp_b200 import blas as B
    torch.cuda.set_device(0)
    m, n, k = 128, 256, 1 << 20
    g = torch.Generator(device="cuda").manual_seed(1)
    A = (torch.randn(m, k, device="cuda", generator=g) / 1024).to(torch.bfloat16)   # stored k x m (OP_T)
    Bm = (torch.randn(n, k, device="cuda", generator=g) / 1024).to(torch.bfloat16)  # stored k x n
    C = torch.zeros(n, m, device="cuda", dtype=torch.float32)
    with B.Handle() as h:
        assert h.gemm_ex(1, 0, m, n, k, 1.0, A, N.GRX_R_16BF, k, Bm, N.GRX_R_16BF, k, 0.0, C, N.GRX_R_32F,
                         m) == N.SUCCESS
        torch.cuda.synchronize()
        first = h.execution_status()
        # the same handle, a problem whose waits all end well inside 1 ms
        a = torch.randn(256, 512, device="cuda", generator=g).to(torch.bfloat16)
        b = torch.randn(384, 512, device="cuda", generator=g).to(torch.bfloat16)
        c = torch.zeros(384, 256, device="cuda", dtype=torch.float32)
        assert h.gemm_ex(1, 0, 256, 384, 512, 1.0, a, N.GRX_R_16BF, 512, b, N.GRX_R_16BF, 512, 0.0, c, N.GRX_R_32F,
                         256) == N.SUCCESS
        torch.cuda.synchronize()
        second = h.execution_status()
        ref = (b.float() @ a.float().T)
        ok = bool(torch.allclose(c, ref, atol=1e-2, rtol=1e-2))
    print(f"RESULT {first} {second} {int(ok)}")
""")


def test_gemm_kernel_abort_path_in_a_real_launch(dev):
    env = dict(os.environ, GRX_WAIT_TIMEOUT_MS="1", GRX_GEMM_SPLITK="0", GRX_GEMM_NO_PAIR="1")
    r = subprocess.run([sys.executable, "-c", CHILD, str(ROOT)], capture_output=True, text=True, timeout=300, env=env)
    line = [ln for ln in r.stdout.splitlines() if ln.startswith("RESULT")]
    assert r.returncode == 0 and line, r.stdout + r.stderr
    first, second, ok = (int(v) for v in line[0].split()[1:])
    assert first == N.EXECUTION_FAILED, "the 7 ms tile should have outlived a 1 ms wait limit"
    assert second == N.SUCCESS and ok == 1, "the next GemmEx after an abort must be correct"
