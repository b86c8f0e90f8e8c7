"""The sharded hot path on real GPUs with NCCL: one process per GPU (2 ranks).

Column-parallel bf16 GemmEx (+ bias) with the all-gather that replicates C,
and (batch*head)-parallel causal attention with its gather, each compared
with the same call made unsharded on rank 0's GPU. Skipped with fewer than
2 GPUs. NVLS is off (NCCL_NVLS_ENABLE=0) and no kernel here uses multicast."""
import os
import socket
import time

import pytest
import torch

pytestmark = pytest.mark.gpu


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    import math

    import torch.distributed as dist

    from grxcp_b200 import _native as N
    from grxcp_b200 import blas as B
    from grxcp_b200 import dnn as D
    from grxcp_b200 import shard as S

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    try:
        g = torch.Generator().manual_seed(3)  # CPU generator: identical inputs on every rank
        m, n, k = 512, 1024, 768
        A = (torch.randn(m * k, generator=g) / math.sqrt(k)).to(torch.bfloat16).to(dev)
        Bm = (torch.randn(k * n, generator=g) / math.sqrt(k)).to(torch.bfloat16).to(dev)
        bias = (torch.randn(n, generator=g) * 0.02).to(dev)
        C = torch.zeros(m * n, device=dev, dtype=torch.bfloat16)
        with B.Handle() as h:
            st = S.gemm_ex_column_parallel(h, N.OP_T, N.OP_N, m, n, k, 1.0, A, N.GRX_R_16BF, k, Bm, N.GRX_R_16BF,
                                           k, 0.0, C, N.GRX_R_16BF, m, bias=bias, rank=rank, world=world,
                                           gather=True)
            assert st == N.SUCCESS
            ref = torch.zeros_like(C)
            h.set_epilogue(bias=bias, bias_type=N.GRX_R_32F)
            assert h.gemm_ex(N.OP_T, N.OP_N, m, n, k, 1.0, A, N.GRX_R_16BF, k, Bm, N.GRX_R_16BF, k, 0.0, ref,
                             N.GRX_R_16BF, m) == N.SUCCESS
            torch.cuda.synchronize()
            assert h.execution_status() == N.SUCCESS
        assert torch.equal(C, ref), "sharded GEMM differs from the unsharded call"

        q_ = torch.randn(2, 4, 384, 128, generator=g).to(torch.bfloat16).to(dev)
        k_ = torch.randn(2, 4, 384, 128, generator=g).to(torch.bfloat16).to(dev)
        v_ = torch.randn(2, 4, 384, 128, generator=g).to(torch.bfloat16).to(dev)
        o = torch.zeros_like(q_)
        lse = torch.zeros(2, 4, 384, device=dev)
        with D.Handle() as dh:
            assert S.attention_head_parallel(dh, q_, k_, v_, o, 1 / math.sqrt(128), True, lse, rank=rank,
                                             world=world, gather=True) == N.SUCCESS
            o_ref = torch.zeros_like(q_)
            l_ref = torch.zeros_like(lse)
            assert dh.attention(q_, k_, v_, o_ref, 1 / math.sqrt(128), True, l_ref) == N.SUCCESS
            torch.cuda.synchronize()
        if not (torch.equal(o, o_ref) and torch.equal(lse, l_ref)):
            do = (o.float() - o_ref.float()).abs().reshape(world, -1).amax(1).tolist()
            dl = (lse - l_ref).abs().reshape(world, -1).amax(1).tolist()
            raise AssertionError(f"sharded attention differs: o per-rank-half {do}, lse {dl}")
        q.put((rank, "ok"))
    except BaseException as e:
        q.put((rank, repr(e)))
    finally:
        dist.destroy_process_group()


def test_sharded_gemm_and_attention_two_gpus():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = {}
    deadline = time.monotonic() + 240
    while len(out) < 2 and time.monotonic() < deadline:
        try:
            r, msg = q.get(timeout=1)
            out[r] = msg
        except Exception:
            pass
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    assert out == {0: "ok", 1: "ok"}, out


def _fused_worker(rank, world, port, q):
    import math

    import torch.distributed as dist

    from grxcp_b200 import _native as N
    from grxcp_b200 import blas as B
    from grxcp_b200 import shard as S

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    cbuf = None
    try:
        for (m, n, k) in [(512, 1024, 768), (4096, 8192, 4096)]:
            g = torch.Generator().manual_seed(7)
            A = (torch.randn(m * k, generator=g) / math.sqrt(k)).to(torch.bfloat16).to(dev)
            Bm = (torch.randn(k * n, generator=g) / math.sqrt(k)).to(torch.bfloat16).to(dev)
            bias = (torch.randn(n, generator=g) * 0.02).to(dev)
            cbuf = S.PeerBuffer(m * n * 2, rank, world)
            Cf = cbuf.local(torch.bfloat16)
            Cf.fill_(float("nan"))
            torch.cuda.synchronize()
            dist.barrier()
            with B.Handle() as h:
                st = S.gemm_ex_column_parallel_fused(h, N.OP_T, N.OP_N, m, n, k, 1.0, A, N.GRX_R_16BF, k, Bm,
                                                     N.GRX_R_16BF, k, 0.0, cbuf, N.GRX_R_16BF, m, bias=bias,
                                                     rank=rank, world=world)
                assert st == N.SUCCESS, N.STATUS.get(st, st)
                assert h.execution_status() == N.SUCCESS
                Cn = torch.zeros(m * n, device=dev, dtype=torch.bfloat16)
                assert S.gemm_ex_column_parallel(h, N.OP_T, N.OP_N, m, n, k, 1.0, A, N.GRX_R_16BF, k, Bm,
                                                 N.GRX_R_16BF, k, 0.0, Cn, N.GRX_R_16BF, m, bias=bias, rank=rank,
                                                 world=world, gather=True) == N.SUCCESS
                torch.cuda.synchronize()
                if not torch.equal(Cf, Cn):
                    raise AssertionError(f"fused replicated C differs from the all-gather path ({m}x{n}x{k})")
                if m == 4096:
                    def timed(fn, it=10):
                        for _ in range(3):
                            fn()
                        torch.cuda.synchronize()
                        dist.barrier()
                        t0 = time.perf_counter()
                        for _ in range(it):
                            fn()
                        torch.cuda.synchronize()
                        return (time.perf_counter() - t0) / it * 1e3
                    tf = timed(lambda: S.gemm_ex_column_parallel_fused(
                        h, N.OP_T, N.OP_N, m, n, k, 1.0, A, N.GRX_R_16BF, k, Bm, N.GRX_R_16BF, k, 0.0, cbuf,
                        N.GRX_R_16BF, m, bias=bias, rank=rank, world=world))
                    tn = timed(lambda: (S.gemm_ex_column_parallel(
                        h, N.OP_T, N.OP_N, m, n, k, 1.0, A, N.GRX_R_16BF, k, Bm, N.GRX_R_16BF, k, 0.0, Cn,
                        N.GRX_R_16BF, m, bias=bias, rank=rank, world=world, gather=True), dist.barrier()))
                    if rank == 0:
                        print(f"replicated C {m}x{n}x{k} on {world} GPUs: fused {tf:.3f} ms, GEMM + all-gather "
                              f"{tn:.3f} ms (wall clock per call incl. barrier)", flush=True)
            dist.barrier()
            cbuf.close()
            cbuf = None
        q.put((rank, "ok"))
    except BaseException as e:
        q.put((rank, repr(e)))
    finally:
        dist.destroy_process_group()


def test_fused_replicated_gemm_two_gpus():
    """Column-parallel GemmEx whose epilogue stores each rank's columns into every rank's copy of C
    (IPC-opened peer buffers, NVLink stores): C equals the GEMM + NCCL all-gather path bit for bit."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_fused_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = {}
    deadline = time.monotonic() + 240
    while len(out) < 2 and time.monotonic() < deadline:
        try:
            r, msg = q.get(timeout=1)
            out[r] = msg
        except Exception:
            pass
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    assert out == {0: "ok", 1: "ok"}, out
