"""Column-parallel GemmEx through the C-ABI (grxblasShard* / grxblasGemmExColumnParallel).

One process per GPU; the parent makes the NCCL unique id (grxblasShardGetUniqueId)
and hands it to the ranks, as a C caller would over a socket. The 1-GPU case
(world 1) runs on any box; the 2-GPU cases are skipped with fewer GPUs:
  * the replicated result on every rank is bit-identical to one unsharded
    grxblasGemmEx with the same epilogue (bias over columns), ragged n included;
  * a rank that leaves between steps: the survivor's next replicated call ends
    with EXECUTION_FAILED within GRX_SHARD_TIMEOUT_MS (the communicator is
    aborted on the host), and its GPU keeps working.
NVLS is off in every rank (NCCL_NVLS_ENABLE=0) and no kernel uses multicast."""
import math
import os
import time

import pytest
import torch

from grxcp_b200 import _native as N
from grxcp_b200 import blas as B

pytestmark = pytest.mark.gpu


def _inputs(m, n, k, dev):
    g = torch.Generator().manual_seed(17)  # CPU generator: the same inputs on every rank
    A = (torch.randn(m * k, generator=g) / math.sqrt(k)).to(torch.bfloat16).to(dev)
    Bm = (torch.randn(k * n, generator=g) / math.sqrt(k)).to(torch.bfloat16).to(dev)
    bias = (torch.randn(n, generator=g) * 0.02).to(dev)
    return A, Bm, bias


def _reference(h, m, n, k, A, Bm, bias):
    ref = torch.zeros(m * n, device=A.device, dtype=torch.bfloat16)
    B.check(h.set_epilogue(bias=bias, bias_type=N.GRX_R_32F))
    B.check(h.gemm_ex(N.OP_T, N.OP_N, m, n, k, 1.0, A, N.GRX_R_16BF, k, Bm, N.GRX_R_16BF, k, 0.0, ref, N.GRX_R_16BF,
                      m))
    torch.cuda.synchronize()
    return ref


def test_column_parallel_world_one(dev):
    st, uid = B.shard_unique_id()
    assert st == N.SUCCESS
    comm = B.ShardComm(uid, 0, 1)
    assert comm.status == N.SUCCESS
    m, n, k = 384, 520, 256
    A, Bm, bias = _inputs(m, n, k, dev)
    C = torch.zeros(m * n, device=dev, dtype=torch.bfloat16)
    with B.Handle() as h:
        ref = _reference(h, m, n, k, A, Bm, bias)
        assert comm.gemm_ex_column_parallel(h, N.OP_T, N.OP_N, m, n, k, 1.0, A, N.GRX_R_16BF, k, Bm, N.GRX_R_16BF, k,
                                            0.0, C, N.GRX_R_16BF, m, True) == N.SUCCESS
        assert comm.synchronize(h) == N.SUCCESS
    assert torch.equal(C, ref)
    assert comm.destroy() == N.SUCCESS


def _rank(rank, world, uid, n, mode, q, go):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    os.environ["GRX_SHARD_TIMEOUT_MS"] = "8000"
    try:
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        from grxcp_b200 import _native as N
        from grxcp_b200 import blas as B

        comm = B.ShardComm(uid, rank, world)
        assert comm.status == N.SUCCESS, f"comm init {comm.status}"
        m, k = 512, 768
        A, Bm, bias = _inputs(m, n, k, dev)
        C = torch.zeros(m * n, device=dev, dtype=torch.bfloat16)
        with B.Handle() as h:
            ref = _reference(h, m, n, k, A, Bm, bias)
            st = comm.gemm_ex_column_parallel(h, N.OP_T, N.OP_N, m, n, k, 1.0, A, N.GRX_R_16BF, k, Bm, N.GRX_R_16BF,
                                              k, 0.0, C, N.GRX_R_16BF, m, True)
            assert st == N.SUCCESS, f"column parallel {st}"
            assert comm.synchronize(h) == N.SUCCESS
            assert torch.equal(C, ref), "replicated C differs from the unsharded GemmEx"
            if mode == "leave":
                if rank == 1:
                    q.put((rank, "ok"))
                    return  # leaves between steps: no destroy, no further collective
                go.wait(60)  # rank 1 has gone
                time.sleep(1.0)
                t0 = time.monotonic()
                st = comm.gemm_ex_column_parallel(h, N.OP_T, N.OP_N, m, n, k, 1.0, A, N.GRX_R_16BF, k, Bm,
                                                  N.GRX_R_16BF, k, 0.0, C, N.GRX_R_16BF, m, True)
                if st == N.SUCCESS:
                    st = comm.synchronize(h)
                waited = time.monotonic() - t0
                assert st == N.EXECUTION_FAILED, f"expected EXECUTION_FAILED after the peer left, got {st}"
                assert waited < 60, waited
                # the aborted communicator refuses further work; the GPU still computes
                assert comm.synchronize(h) == N.EXECUTION_FAILED
                C2 = torch.zeros_like(C)
                B.check(h.gemm_ex(N.OP_T, N.OP_N, m, n, k, 1.0, A, N.GRX_R_16BF, k, Bm, N.GRX_R_16BF, k, 0.0, C2,
                                  N.GRX_R_16BF, m))
                torch.cuda.synchronize()
                assert h.execution_status() == N.SUCCESS
                assert torch.equal(C2, ref)
        assert comm.destroy() == N.SUCCESS
        q.put((rank, "ok"))
    except BaseException as e:  # noqa: BLE001
        q.put((rank, repr(e)))


def _run_two(n, mode):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp

    st, uid = B.shard_unique_id()
    assert st == N.SUCCESS
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    go = ctx.Event()
    procs = [ctx.Process(target=_rank, args=(r, 2, uid, n, mode, q, go)) for r in range(2)]
    for p in procs:
        p.start()
    out = {}
    deadline = time.monotonic() + 240
    while len(out) < 2 and time.monotonic() < deadline:
        try:
            r, msg = q.get(timeout=1)
            out[r] = msg
            if mode == "leave" and r == 1:
                procs[1].join(30)
                go.set()
        except Exception:  # noqa: BLE001
            pass
    for p in procs:
        p.join(30)
        if p.is_alive():
            p.kill()
    assert out == {0: "ok", 1: "ok"}, out


def test_column_parallel_two_gpus_replicated():
    _run_two(1000, "equal")  # 1000 columns: 500 each; ragged tiles at the seam


def test_column_parallel_two_gpus_ragged_split():
    _run_two(777, "equal")  # 389 + 388 columns


def test_column_parallel_peer_leaves_between_steps():
    _run_two(1024, "leave")
