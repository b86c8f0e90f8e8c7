"""Host-side fault injection (GRX_FAULT_INJECT), CPU part.

Failure detection is tested without a GPU fault: the library is told that a
host-side call failed, and the API must return the status a real failure of
that call returns. Sites that fail before any device is touched are tested
here; tests/test_fault_injection_gpu.py covers the device allocations and the
kernel-path resolution on a GPU."""
import pytest

from grxcp_b200 import _native as N
from grxcp_b200 import blas as B


def test_shard_range_matches_python_rule():
    from grxcp_b200.shard import even_shard

    for n in (0, 1, 7, 1000, 1024):
        for world in (1, 2, 3, 8):
            total = 0
            for r in range(world):
                st, s, c = B.shard_range(n, r, world)
                e = even_shard(n, world, r)
                assert st == N.SUCCESS and (s, c) == (e.start, e.count)
                total += c
            assert total == n
    assert B.shard_range(10, 2, 2)[0] == N.INVALID_VALUE
    assert B.shard_range(-1, 0, 2)[0] == N.INVALID_VALUE


def test_nccl_init_failure_is_execution_failed(monkeypatch):
    monkeypatch.setenv("GRX_FAULT_INJECT", "nccl_init")
    comm = B.ShardComm(b"\0" * 128, 0, 2)
    assert comm.status == N.EXECUTION_FAILED
    assert not comm.c  # no communicator handed out


def test_nccl_missing_is_not_supported(monkeypatch):
    monkeypatch.setenv("GRX_FAULT_INJECT", "alloc,nccl_load")
    assert B.ShardComm(b"\0" * 128, 0, 2).status == N.NOT_SUPPORTED
    assert B.shard_unique_id()[0] == N.NOT_SUPPORTED


def test_shard_argument_refusals():
    assert B.ShardComm(b"\0" * 128, 2, 2).status == N.INVALID_VALUE
    assert B.ShardComm(b"\0" * 128, 0, 0).status == N.INVALID_VALUE
    with B.Handle() as h:
        st = N.lib.grxblasGemmExColumnParallel(h.h, None, 0, 0, 8, 8, 8, None, None, N.GRX_R_16BF, 8, None,
                                               N.GRX_R_16BF, 8, None, None, N.GRX_R_16BF, 8, 1)
        assert st == N.INVALID_VALUE  # no communicator
    st = N.lib.grxblasGemmExColumnParallel(None, None, 0, 0, 8, 8, 8, None, None, N.GRX_R_16BF, 8, None,
                                           N.GRX_R_16BF, 8, None, None, N.GRX_R_16BF, 8, 1)
    assert st == N.NOT_INITIALIZED


@pytest.mark.parametrize("site", ["alloc", "module"])
def test_injection_list_parsing(monkeypatch, site):
    # an unrelated list entry must not trip the site, the exact name must
    monkeypatch.setenv("GRX_FAULT_INJECT", "allocx,xmodule,nccl")
    assert B.ShardComm(b"\0" * 128, 2, 2).status == N.INVALID_VALUE
    monkeypatch.setenv("GRX_FAULT_INJECT", f"nccl_init,{site}")
    assert B.ShardComm(b"\0" * 128, 0, 2).status == N.EXECUTION_FAILED
