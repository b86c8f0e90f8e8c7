"""Multi-GPU sharding of the hot path: one process per GPU, torch.distributed.

The reference has no multi-device compute (peer access is refused,
src/runtime/context.cpp:401-410), so this layer is new. It follows the two
natural partitions of the path:

* GEMM, column-parallel over N. With column-major storage the columns
  [j0, j1) of op(B) and of C are contiguous (OP_N B: B + j0*ldb; OP_T B is
  stored n x k, so its rows j0.. start at B + j0), and so is bias[j0:j1]. Each
  rank holds all of A and its own columns, and runs one local grxblasGemmEx:
  no collective on the data path. When the caller wants C replicated on every
  rank, one NCCL all-gather of the equal contiguous chunks assembles it.
* Attention, over the flattened batch*heads index: rank r owns a contiguous
  range of (b, h) pairs and computes their O and LSE; an optional all-gather
  replicates them.

Everything here is plumbing around the library's C-ABI calls; the GEMM and
attention themselves run in libgrxcp.so. `check_peers` lets ranks notice a
peer that stopped (died or hung between steps) from a heartbeat in the
torch.distributed store, instead of blocking in the next collective.
"""
from __future__ import annotations

import time
from dataclasses import dataclass

from . import _native as N


@dataclass(frozen=True)
class Shard:
    start: int
    count: int

    @property
    def stop(self) -> int:
        return self.start + self.count


def even_shard(total: int, world: int, rank: int) -> Shard:
    """Contiguous split of `total` units over `world` ranks; the first
    total % world ranks get one more unit (all chunks equal when it divides)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("bad world/rank")
    base, extra = divmod(total, world)
    start = rank * base + min(rank, extra)
    return Shard(start, base + (1 if rank < extra else 0))


def column_views(B, C, bias, transb: int, ldb: int, ldc: int, cols: Shard):
    """Views of this rank's columns of op(B), C (column-major, flat 1-D tensors)
    and bias. Returns (B_view, C_view, bias_view)."""
    if transb == N.OP_N:
        b = B[cols.start * ldb:]
    else:
        b = B[cols.start:]
    c = C[cols.start * ldc: cols.stop * ldc]
    bv = None if bias is None else bias[cols.start:cols.stop]
    return b, c, bv


def gemm_ex_column_parallel(handle, transa, transb, m, n, k, alpha, A, Atype, lda, B, Btype, ldb, beta, C, Ctype,
                            ldc, bias=None, rank: int = 0, world: int = 1, gather: bool = False, group=None) -> int:
    """This rank's share of C = alpha*op(A)op(B) + beta*C (+ bias): one local
    grxblasGemmEx over columns even_shard(n, world, rank). A and the full-size B,
    C, bias are flat 1-D tensors (B/C/bias need only hold this rank's columns
    at their global offsets). With gather=True, C ends up complete on every rank
    (NCCL all-gather; requires n % world == 0 so the chunks are equal and
    contiguous). Returns the GemmEx status."""
    cols = even_shard(n, world, rank)
    b, c, bv = column_views(B, C, bias, transb, ldb, ldc, cols)
    if bias is not None:
        st = handle.set_epilogue(bias=bv, bias_type=N.GRX_R_32F if bias.dtype.itemsize == 4 else N.GRX_R_16BF)
        if st != N.SUCCESS:
            return st
    st = N.SUCCESS
    if cols.count > 0:
        st = handle.gemm_ex(transa, transb, m, cols.count, k, alpha, A, Atype, lda, b, Btype, ldb, beta, c, Ctype,
                            ldc)
    if bias is not None:
        handle.clear_epilogue()
    if st == N.SUCCESS and gather and world > 1:
        if n % world:
            raise ValueError("gather needs n divisible by the world size")
        all_gather_chunks(C, ldc * (n // world), rank, world, group)
    return st


class _CudaArray:
    """A raw device range as a torch-importable object (CUDA array interface)."""

    def __init__(self, ptr: int, numel: int, typestr: str):
        self.__cuda_array_interface__ = {"shape": (numel,), "typestr": typestr, "data": (ptr, False), "version": 3,
                                         "strides": None}


class PeerBuffer:
    """One device buffer per rank, each opened in every rank's process.

    The buffer is a grxMalloc allocation (a whole allocation, as CUDA IPC
    requires); its IPC handle is exchanged through the process group and every
    peer's copy is opened with grxIpcOpenMemHandle. `ptrs[r]` is rank r's copy
    as a device address valid in this process; `local(dtype)` is this rank's
    copy as a flat torch tensor. Collective: every rank constructs it with the
    same size."""

    def __init__(self, nbytes: int, rank: int, world: int, group=None):
        import ctypes as C

        import torch.distributed as dist

        self.rank, self.world, self.nbytes = rank, world, nbytes
        p = C.c_void_p()
        st = N.lib.grxMalloc(C.byref(p), nbytes)
        if st != 0 or not p.value:
            raise RuntimeError(f"grxMalloc({nbytes}) failed: {st}")
        self._own = p.value
        h = N.grxIpcMemHandle_t()
        st = N.lib.grxIpcGetMemHandle(C.byref(h), C.c_void_p(self._own))
        if st != 0:
            raise RuntimeError(f"grxIpcGetMemHandle failed: {st}")
        handles = [None] * world
        dist.all_gather_object(handles, bytes(h.reserved), group=group)
        self.ptrs = []
        self._opened = []
        for r in range(world):
            if r == rank:
                self.ptrs.append(self._own)
                continue
            hr = N.grxIpcMemHandle_t()
            C.memmove(hr.reserved, handles[r], 64)
            q = C.c_void_p()
            st = N.lib.grxIpcOpenMemHandle(C.byref(q), hr)
            if st != 0 or not q.value:
                raise RuntimeError(f"grxIpcOpenMemHandle(rank {r}) failed: {st}")
            self.ptrs.append(q.value)
            self._opened.append(q.value)

    def local(self, dtype):
        """This rank's copy as a flat torch tensor of `dtype` (bf16, fp16 or fp32)."""
        import torch

        es = torch.tensor([], dtype=dtype).element_size()
        code = {4: "<f4", 2: "<i2"}[es]
        t = torch.as_tensor(_CudaArray(self._own, self.nbytes // es, code), device="cuda")
        return t.view(dtype)

    def close(self) -> None:
        for q in self._opened:
            N.lib.grxIpcCloseMemHandle(q)
        self._opened = []
        if self._own:
            N.lib.grxFree(self._own)
            self._own = 0


def gemm_ex_column_parallel_fused(handle, transa, transb, m, n, k, alpha, A, Atype, lda, B, Btype, ldb, beta,
                                  cbuf: PeerBuffer, Ctype, ldc, bias=None, rank: int = 0, world: int = 1,
                                  group=None) -> int:
    """Column-parallel GemmEx whose epilogue writes this rank's columns into
    every rank's copy of C (cbuf, a PeerBuffer holding the full ldc x n C):
    the replicated-output step fused into the GEMM over NVLink instead of a
    separate all-gather. 16-bit inputs only (grxblasSetPeerOutputs).

    Ordering: the call starts with a barrier (after this rank's stream has
    drained), so no peer stores into this rank's C while this rank may still
    be reading the previous contents, and ends with a device synchronise
    followed by a barrier, so on return C is complete on every rank whatever
    the process group's backend (a gloo barrier does not order GPU work)."""
    import torch
    import torch.distributed as dist

    cols = even_shard(n, world, rank)
    es = 4 if Ctype == N.GRX_R_32F else 2
    C = cbuf.local(torch.float32 if es == 4 else (torch.bfloat16 if Ctype == N.GRX_R_16BF else torch.float16))
    b, c, bv = column_views(B, C, bias, transb, ldb, ldc, cols)
    off = cols.start * ldc * es
    st = handle.set_peer_outputs([cbuf.ptrs[r] + off for r in range(world) if r != rank])
    if st != N.SUCCESS:
        return st
    if bias is not None:
        st = handle.set_epilogue(bias=bv, bias_type=N.GRX_R_32F if bias.dtype.itemsize == 4 else N.GRX_R_16BF)
        if st != N.SUCCESS:
            return st
    if world > 1:
        # Entry barrier: every rank has finished with cbuf's previous contents.
        torch.cuda.synchronize()
        dist.barrier(group=group)
    try:
        if cols.count > 0:
            st = handle.gemm_ex(transa, transb, m, cols.count, k, alpha, A, Atype, lda, b, Btype, ldb, beta, c, Ctype,
                                ldc)
    finally:
        handle.set_peer_outputs([])
        if bias is not None:
            handle.clear_epilogue()
    if world > 1:
        # This rank's kernel, and its stores into the other copies, completes
        # before the rank enters the barrier. Entered on failure too, so that
        # no rank is left waiting for one that returned early.
        torch.cuda.synchronize()
        dist.barrier(group=group)
    return st


def all_gather_chunks(flat, chunk: int, rank: int, world: int, group=None) -> None:
    """flat holds `world` equal contiguous chunks; chunk `rank` is this rank's.
    After the call every rank holds all of them (NCCL on CUDA tensors, the list
    form of all_gather on gloo CPU ranks)."""
    import torch.distributed as dist

    if flat.numel() < chunk * world:
        raise ValueError("buffer smaller than world * chunk")
    mine = flat[rank * chunk:(rank + 1) * chunk].clone()
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(flat[:chunk * world], mine, group=group)
    else:
        parts = list(flat[:chunk * world].split(chunk))
        dist.all_gather(parts, mine, group=group)


def attention_head_parallel(dnn_handle, q, k, v, o, scale: float, causal: bool, lse=None, rank: int = 0,
                            world: int = 1, gather: bool = False, group=None) -> int:
    """This rank's (batch*head) range of attention forward. q/k/v/o are
    [B, H, S, D] contiguous tensors present on every rank (only this rank's
    range is read / written); lse is [B, H, S] or None."""
    B_, H, S, D = q.shape
    bh = even_shard(B_ * H, world, rank)
    st = N.SUCCESS
    if bh.count > 0:
        qf = q.reshape(B_ * H, S, D)[bh.start:bh.stop].unsqueeze(0)
        kf = k.reshape(B_ * H, k.shape[2], D)[bh.start:bh.stop].unsqueeze(0)
        vf = v.reshape(B_ * H, v.shape[2], D)[bh.start:bh.stop].unsqueeze(0)
        of = o.reshape(B_ * H, S, D)[bh.start:bh.stop].unsqueeze(0)
        lf = None if lse is None else lse.reshape(B_ * H, S)[bh.start:bh.stop]
        st = dnn_handle.attention(qf, kf, vf, of, scale, causal, lf)
    if st == N.SUCCESS and gather and world > 1:
        if (B_ * H) % world:
            raise ValueError("gather needs batch*heads divisible by the world size")
        all_gather_chunks(o.view(-1), (B_ * H // world) * S * D, rank, world, group)
        if lse is not None:
            all_gather_chunks(lse.view(-1), (B_ * H // world) * S, rank, world, group)
    return st


class PeerFailure(RuntimeError):
    pass


def heartbeat(store, rank: int, step: int) -> None:
    """Record that `rank` finished `step` (call between steps, with no kernel
    or collective of this rank in flight)."""
    store.set(f"grxcp/hb/{rank}", str(step))


def check_peers(store, rank: int, world: int, step: int, timeout_s: float = 5.0, poll_s: float = 0.05) -> None:
    """Wait until every peer has reported `step` (or later) via heartbeat().
    Raises PeerFailure naming the ranks that did not within `timeout_s`, so a
    rank that died or hung between steps is noticed on the host before the next
    launch rather than inside a blocking collective."""
    deadline = time.monotonic() + timeout_s
    missing = [r for r in range(world) if r != rank]
    while missing:
        still = []
        for r in missing:
            key = f"grxcp/hb/{r}"
            try:
                ok = store.check([key]) and int(store.get(key)) >= step
            except Exception:
                ok = False
            if not ok:
                still.append(r)
        missing = still
        if not missing:
            return
        if time.monotonic() > deadline:
            raise PeerFailure(f"rank {rank}: no heartbeat for step {step} from rank(s) {missing}")
        time.sleep(poll_s)
