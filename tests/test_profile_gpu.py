"""GRX_PROFILE tracing: the reference's GRXPROF line contract
(src/runtime/profile.cpp:147-290) from the library's own launches. A child
process runs a GEMM and an RMSNorm with GRX_PROFILE=1; its stderr must hold one
device line and one op=launch line per kernel launch, each with the kernel
name, grid/block/shared and a positive device time. Without the variable the
same run prints no GRXPROF line."""
import os
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parent.parent

CHILD = r"""
import sys; sys.path.insert(0, %r)
import torch
from grxcp_b200 import blas as B, dnn as D, _native as N
a = torch.randn(256 * 256, device="cuda").to(torch.bfloat16)
c = torch.empty(256 * 256, device="cuda", dtype=torch.bfloat16)
with B.Handle() as h:
    assert h.gemm_ex(1, 0, 256, 256, 256, 1.0, a, N.GRX_R_16BF, 256, a, N.GRX_R_16BF, 256, 0.0, c, N.GRX_R_16BF, 256) == 0
x = torch.randn(64, 4096, device="cuda").to(torch.bfloat16)
g = torch.ones(4096, device="cuda")
with D.Handle() as d:
    assert d.rmsnorm(x, g, 1e-5, torch.empty_like(x)) == 0
torch.cuda.synchronize()
""" % str(ROOT)


def _run(env_extra):
    env = dict(os.environ)
    env.pop("GRX_PROFILE", None)
    env.update(env_extra)
    r = subprocess.run([sys.executable, "-c", CHILD], env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    return [l for l in r.stderr.splitlines() if l.startswith("GRXPROF|")]


def test_grxprof_lines():
    lines = _run({"GRX_PROFILE": "1"})
    dev = [l for l in lines if l.startswith("GRXPROF|device|")]
    launches = [l for l in lines if l.startswith("GRXPROF|1|op=launch|")]
    assert len(dev) == 1 and "event_timing_is_device_side=1" in dev[0]
    kv = [dict(f.split("=", 1) for f in l.split("|")[2:]) for l in launches]
    names = [k["kernel"] for k in kv]
    assert any(n.startswith("tc_gemm") for n in names) and "norm_vec_kernel" in names
    for k in kv:
        assert int(k["c.device_ns"]) > 0
        assert int(k["host_end_ns"]) >= int(k["host_start_ns"])
        assert k["module"].endswith("libgrxcp.so")
        assert len(k["grid"].split(".")) == 3 and len(k["block"].split(".")) == 3
    assert [int(k["seq"]) for k in kv] == list(range(len(kv)))


def test_no_trace_by_default():
    assert _run({}) == []
