"""The multi-GPU layer's host logic on CPU: world-size-2 gloo ranks.

The GEMM / attention kernels cannot run here, so each rank's local call goes to
a stand-in handle that computes its shard with the oracle; what is under test
is the sharding (column / (batch, head) ranges and pointer views), the
all-gather that replicates the result, and failure detection (a rank that
stops between steps is reported by its peers from the store heartbeat)."""
from __future__ import annotations

import os
import socket
import time

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from grxcp_b200 import _native as N
from grxcp_b200 import shard as S


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _init(rank, world, port):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)


class OracleBlas:
    """Stand-in for grxblas.Handle on CPU tensors (fp32 values, fp64 oracle)."""

    def __init__(self):
        self.bias = None

    def set_epilogue(self, bias=None, bias_type=None, **kw):
        self.bias = bias
        return N.SUCCESS

    def clear_epilogue(self):
        self.bias = None
        return N.SUCCESS

    def gemm_ex(self, ta, tb, m, n, k, alpha, A, at, lda, B, bt, ldb, beta, C, ct, ldc):
        out = oracle.gemm_f64(ta, tb, m, n, k, alpha, A.numpy(), lda, B.numpy(), ldb,
                              bias=None if self.bias is None else self.bias.numpy(), ldc=ldc)
        C[: ldc * n] = torch.from_numpy(out[: ldc * n].astype(np.float32))
        return N.SUCCESS


class OracleDnn:
    def attention(self, q, k, v, o, scale, causal, lse=None):
        ro, rl = oracle.attention(q[0].numpy(), k[0].numpy(), v[0].numpy(), scale, causal)
        o[0].copy_(torch.from_numpy(ro.astype(np.float32)))
        if lse is not None:
            lse.copy_(torch.from_numpy(rl.astype(np.float32)))
        return N.SUCCESS


def _gemm_worker(rank, world, port, q):
    _init(rank, world, port)
    try:
        rng = np.random.default_rng(0)
        for ta, tb in [(1, 0), (0, 1)]:
            m, n, k = 24, 32, 20
            A = torch.from_numpy(rng.standard_normal(m * k).astype(np.float32))
            Bm = torch.from_numpy(rng.standard_normal(k * n).astype(np.float32))
            bias = torch.from_numpy(rng.standard_normal(n).astype(np.float32))
            lda, ldb = (k if ta else m), (n if tb else k)
            C = torch.zeros(m * n)
            st = S.gemm_ex_column_parallel(OracleBlas(), ta, tb, m, n, k, 1.0, A, N.GRX_R_32F, lda, Bm, N.GRX_R_32F,
                                           ldb, 0.0, C, N.GRX_R_32F, m, bias=bias, rank=rank, world=world,
                                           gather=True)
            assert st == N.SUCCESS
            want = oracle.gemm_f64(ta, tb, m, n, k, 1.0, A.numpy(), lda, Bm.numpy(), ldb, bias=bias.numpy())
            assert np.allclose(C.numpy(), want, rtol=1e-5, atol=1e-5), (rank, ta, tb)
        q.put((rank, "ok"))
    except Exception as e:  # report to the parent instead of hanging
        q.put((rank, repr(e)))
    finally:
        dist.destroy_process_group()


def _attn_worker(rank, world, port, q):
    _init(rank, world, port)
    try:
        g = torch.Generator().manual_seed(1)
        B_, H, Sq, D = 2, 3, 40, 16
        qq = torch.randn(B_, H, Sq, D, generator=g)
        kk = torch.randn(B_, H, Sq, D, generator=g)
        vv = torch.randn(B_, H, Sq, D, generator=g)
        o = torch.zeros_like(qq)
        lse = torch.zeros(B_, H, Sq)
        st = S.attention_head_parallel(OracleDnn(), qq, kk, vv, o, 0.25, True, lse, rank=rank, world=world,
                                       gather=True)
        assert st == N.SUCCESS
        ro, rl = oracle.attention(qq.reshape(6, Sq, D).numpy(), kk.reshape(6, Sq, D).numpy(),
                                  vv.reshape(6, Sq, D).numpy(), 0.25, True)
        assert np.allclose(o.reshape(6, Sq, D).numpy(), ro, atol=1e-5)
        assert np.allclose(lse.reshape(6, Sq).numpy(), rl, atol=1e-5)
        q.put((rank, "ok"))
    except Exception as e:
        q.put((rank, repr(e)))
    finally:
        dist.destroy_process_group()


def _failure_worker(rank, world, port, q):
    _init(rank, world, port)
    store = dist.distributed_c10d._get_default_store()
    try:
        S.heartbeat(store, rank, 0)
        S.check_peers(store, rank, world, 0, timeout_s=10)
        if rank == 1:
            q.put((rank, "left"))
            q.close()
            q.join_thread()  # flush before leaving
            os._exit(0)  # leaves between steps, nothing in flight, no heartbeat for step 1
        S.heartbeat(store, rank, 1)
        t0 = time.monotonic()
        try:
            S.check_peers(store, rank, world, 1, timeout_s=1.0)
            q.put((rank, "missed the failure"))
        except S.PeerFailure as e:
            q.put((rank, "detected" if "[1]" in str(e) and time.monotonic() - t0 < 5 else repr(e)))
    except Exception as e:
        q.put((rank, repr(e)))


def _run(fn, world=2, timeout=120):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=fn, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    deadline = time.monotonic() + timeout
    while len(out) < world and time.monotonic() < deadline:
        try:
            r, msg = q.get(timeout=1)
            out[r] = msg
        except Exception:
            pass
    for p in procs:
        p.join(timeout=10)
        if p.is_alive():
            p.kill()
    return out


def test_even_shard():
    assert [S.even_shard(10, 3, r) for r in range(3)] == [S.Shard(0, 4), S.Shard(4, 3), S.Shard(7, 3)]
    assert S.even_shard(8192, 8, 7) == S.Shard(7168, 1024)
    with pytest.raises(ValueError):
        S.even_shard(8, 2, 2)


def test_column_views():
    B = torch.arange(40)
    C = torch.arange(100)
    b, c, bv = S.column_views(B, C, torch.arange(10), N.OP_N, 4, 10, S.Shard(3, 2))
    assert b[0] == 12 and c[0] == 30 and len(c) == 20 and bv.tolist() == [3, 4]
    b, _, _ = S.column_views(B, C, None, N.OP_T, 10, 10, S.Shard(3, 2))
    assert b[0] == 3


def test_gemm_column_parallel_two_ranks():
    out = _run(_gemm_worker)
    assert out == {0: "ok", 1: "ok"}, out


def test_attention_head_parallel_two_ranks():
    out = _run(_attn_worker)
    assert out == {0: "ok", 1: "ok"}, out


def test_peer_that_leaves_between_steps_is_detected():
    out = _run(_failure_worker)
    assert out.get(1) == "left" and out.get(0) == "detected", out
