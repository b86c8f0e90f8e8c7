"""Benchmark of the grxcp-b200 hot path on B200.

Headline: grxblasGemmEx bf16 x bf16 -> fp32 accumulate ->
bf16, M = N = K = 8192, plus a bias[N] epilogue, alpha = 1, beta = 0, called
through the library's C-ABI. One step = one GEMM over the whole job. At N GPUs
the GEMM is column-sharded over N (each rank owns N/G contiguous columns of B
and C, no collective on the data path), so the total work is fixed: strong
scaling. `value` = whole-job TFLOP/s from the max over ranks of the
CUDA-event time of K steps.

Also reported on the same line: the other BASELINE configs measured on rank 0
(attention, RMSNorm / LayerNorm, fp8 strided-batched MLP GEMM, int8 512^3),
the end-to-end number through the public API with host buffers, the roofline
of the dominant kernel, clocks sampled during the timed region, and the CPU
baseline (the oracle port of the reference's CPU GEMM loop).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

M = N = K = 8192
PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d, "measured"
    return PEAKS_FALLBACK, "fallback"


def dist_env():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


# ------------------------------------------------------------------ clocks

class ClockSampler:
    """nvidia-smi clock / throttle sampling during the timed region."""

    def __init__(self, gpu_index: int):
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--id={gpu_index}", f"--query-gpu={q}",
                                       "--format=csv,noheader,nounits", "-lms", "100"], stdout=self.f,
                                      stderr=subprocess.DEVNULL)
        except Exception:
            self.p = None

    def stop(self) -> dict:
        if self.p is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.p.terminate()
        try:
            self.p.wait(timeout=5)
        except Exception:
            self.p.kill()
        self.f.seek(0)
        rows = [l.split(",") for l in self.f.read().splitlines() if l.strip()]
        os.unlink(self.f.name)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            try:
                sm.append(float(r[1]))
                mx = float(r[2])
                for nm, v in zip(names, r[5:9]):
                    if v.strip().lower() == "active":
                        reasons.add(nm)
            except (ValueError, IndexError):
                continue
        loaded = [s for s in sm if mx and s > 0.5 * mx] or sm
        return {"sm_mhz": statistics.median(loaded) if loaded else None, "sm_max_mhz": mx,
                "samples": len(sm), "reasons": sorted(reasons)}


# ------------------------------------------------------------------ CPU baseline (oracle port)

def cpu_gemm_sample(seconds: float, threads: int):
    """Times the oracle port of the reference's CPU GEMM loop (tests/libs/test_grxblas.cpp:63-80:
    naive triple loop, fp64 accumulate) on a column sample of the 8192^3 config.
    Returns (TFLOP/s, columns, seconds)."""
    import numpy as np

    import oracle

    rng = np.random.default_rng(0)
    A = (rng.standard_normal(M * K, dtype=np.float32) / math.sqrt(K)).astype(np.float32)
    cols = max(threads, 1)
    Bs = (rng.standard_normal(K * cols, dtype=np.float32) / math.sqrt(K)).astype(np.float32)
    out = np.empty(M * cols)
    t0 = time.perf_counter()
    oracle.gemm_f64(1, 0, M, cols, K, 1.0, A, K, Bs, K, out=out, nthreads=threads)
    t1 = time.perf_counter() - t0
    target = max(cols, int(cols * seconds / max(t1, 1e-3)))
    target = min(target, N)
    Bs = (rng.standard_normal(K * target, dtype=np.float32) / math.sqrt(K)).astype(np.float32)
    out = np.empty(M * target)
    t0 = time.perf_counter()
    oracle.gemm_f64(1, 0, M, target, K, 1.0, A, K, Bs, K, out=out, nthreads=threads)
    dt = time.perf_counter() - t0
    return 2.0 * M * K * target / dt / 1e12, target, dt


def run_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return 0
    threads = len(os.sched_getaffinity(0))
    vals = []
    cols = 0
    for s in range(args.warmup + args.steps):
        v, cols, dt = cpu_gemm_sample(2.0, threads)
        if s >= args.warmup:
            vals.append(v)
    value = statistics.median(vals)
    line = {
        "impl": "reference",
        "metric": "GEMM TFLOP/s (% dense tensor peak) at 1/2/4/8 B200; attention TFLOP/s; norm GB/s",
        "value": value, "unit": "TFLOP/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f64",
        "data": "synthetic: A, B ~N(0,1)/sqrt(K), seeded",
        "config": config_dict(args.gpus),
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": threads, "kind": "port",
                         "sample": f"{cols} of {N} output columns of the 8192^3 GEMM per step (fp64 naive loop, "
                                   "oracle restatement of tests/libs/test_grxblas.cpp:63-80)"},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def config_dict(gpus):
    return {"workload": "grxblasGemmEx bf16 in / fp32 acc / bf16 out + bias[N], M=N=K=8192 (BASELINE config 2)",
            "m": M, "n": N, "k": K, "transa": "T", "transb": "N", "alpha": 1.0, "beta": 0.0,
            "parallelism": f"column-shard over N x{gpus}" if gpus > 1 else "single GPU",
            "l2": "inputs larger than L2 (A+B+C = 384 MiB per step)"}


# ------------------------------------------------------------------ GPU arm

def run_gpu(args):
    import torch

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import torch.distributed as dist

        # NCCL may print a banner on stdout during init; keep stdout for the JSON line.
        sys.stdout.flush()
        saved = os.dup(1)
        os.dup2(2, 1)
        try:
            dist.init_process_group("nccl", device_id=dev)
            dist.barrier()
        finally:
            sys.stdout.flush()
            os.dup2(saved, 1)
            os.close(saved)
    from grxcp_b200 import _native as Nn
    from grxcp_b200 import blas as B

    peaks, peaks_src = load_peaks()
    stream = torch.cuda.current_stream()
    h = B.Handle()
    B.check(h.set_stream(stream), "set_stream")

    # column shard of B / C / bias owned by this rank
    assert N % world == 0
    nl = N // world
    g = torch.Generator(device=dev).manual_seed(1234)
    A = (torch.randn(M, K, device=dev, generator=g) / math.sqrt(K)).to(torch.bfloat16)  # stored k x m (OP_T)
    Bfull = torch.empty(N, K, device=dev, dtype=torch.bfloat16)
    Bfull.copy_((torch.randn(N, K, device=dev, generator=g) / math.sqrt(K)).to(torch.bfloat16))
    Bl = Bfull[rank * nl:(rank + 1) * nl].contiguous()  # stored k x nl, column-major
    del Bfull
    bias = (torch.randn(N, device=dev, generator=g) * 0.02)[rank * nl:(rank + 1) * nl].contiguous()
    C = torch.empty(nl, M, device=dev, dtype=torch.bfloat16)  # column-major m x nl
    B.check(h.set_epilogue(bias=bias, bias_type=Nn.GRX_R_32F), "set_epilogue")

    def step():
        s = h.gemm_ex(Nn.OP_T, Nn.OP_N, M, nl, K, 1.0, A, Nn.GRX_R_16BF, K, Bl, Nn.GRX_R_16BF, K, 0.0, C,
                      Nn.GRX_R_16BF, M)
        if s != Nn.SUCCESS:
            raise RuntimeError(f"grxblasGemmEx: {Nn.STATUS[s]}")

    def barrier():
        if world > 1:
            import torch.distributed as dist

            dist.barrier()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        import torch.distributed as dist

        t = torch.tensor([x], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    time.sleep(0.3)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for _ in range(args.steps):
        step()
    ev1.record(stream)
    torch.cuda.synchronize()
    clk = clocks.stop()
    barrier()
    torch.cuda.synchronize()
    ms_local = ev0.elapsed_time(ev1) / args.steps
    ms = max_over_ranks(ms_local)
    flops_total = 2.0 * M * N * K
    value = flops_total / (ms * 1e-3) / 1e12
    st = h.execution_status()
    if st != Nn.SUCCESS:
        raise RuntimeError(f"kernel reported {Nn.STATUS[st]}")

    # per-launch kernel time of the dominant kernel = the step (one launch per step)
    per_launch_flops = 2.0 * M * nl * K
    achieved = per_launch_flops / (ms_local * 1e-3) / 1e12
    peak = peaks["bf16_tflops"]
    # DRAM bytes of one launch of this rank's slice, from an ncu capture of that
    # exact shape (bench.py --profile gemm --profile-cols nl); null when absent.
    traffic = None
    tr = ROOT / "profiles" / "traffic.txt"
    if tr.exists():
        for line in tr.read_text().splitlines():
            parts = line.split()
            if len(parts) == 2 and parts[0] == f"gemm_bf16_{M}x{nl}x{K}_per_launch_bytes":
                traffic = float(parts[1])
    # the library's choice (gemm_tc.cu use_pair): CTA pairs for 16-bit problems with at least one
    # 256 x 256 pair-tile per pair of SMs
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    pair = M >= 256 and nl >= 256 and -(-M // 256) * -(-nl // 256) >= sms // 2
    kernel_name = "grx::tc_gemm_pair_kernel<kind::f16, bf16 out>" if pair else "grx::tc_gemm_kernel<kind::f16, bf16 out>"
    roofline = {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
                "traffic": traffic, "peak_source": f"{peaks_src} bf16_tflops (burst)",
                "kernel": kernel_name}

    # ---- end to end through the public API with host buffers (pinned). Every
    # step copies its inputs host -> device and its result device -> host; the
    # steps are pipelined the way a serving loop would run them: step i+1's
    # uploads (copy stream 1) overlap step i's GEMM (compute stream) and its
    # download (copy stream 2), with double-buffered device tensors.
    # Column-parallel wants A replicated: each rank uploads only its 1/world of
    # A's rows (stored k x m, so a row band of op(A) is contiguous) and one NCCL
    # all-gather over NVLink assembles A in every rank's HBM; host links carry
    # A once per step in total instead of once per rank.
    assert M % world == 0
    mrows = M // world
    hA = A[rank * mrows:(rank + 1) * mrows].cpu().pin_memory()
    hB = Bl.cpu().pin_memory()
    hbias = bias.cpu().pin_memory()
    hC = [torch.empty(nl, M, dtype=torch.bfloat16).pin_memory() for _ in range(2)]
    dA = [torch.empty_like(A) for _ in range(2)]
    dB = [torch.empty_like(Bl) for _ in range(2)]
    dbias = [torch.empty_like(bias) for _ in range(2)]
    dC = [C, torch.empty_like(C)]
    up, down = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
    ev = lambda: torch.cuda.Event()  # noqa: E731
    h2d_done, gemm_done, d2h_done = [ev(), ev()], [ev(), ev()], [ev(), ev()]
    for e in gemm_done + d2h_done:
        e.record(stream)

    def e2e_step(i):
        bsel = i & 1
        with torch.cuda.stream(up):
            up.wait_event(gemm_done[bsel])  # the GEMM that last read these buffers is done
            if world > 1:
                import torch.distributed as dist

                mine = dA[bsel][rank * mrows:(rank + 1) * mrows]
                mine.copy_(hA, non_blocking=True)
                dist.all_gather_into_tensor(dA[bsel], mine)  # on the upload stream (torch's current here)
            else:
                dA[bsel].copy_(hA, non_blocking=True)
            dB[bsel].copy_(hB, non_blocking=True)
            dbias[bsel].copy_(hbias, non_blocking=True)
            h2d_done[bsel].record(up)
        stream.wait_event(h2d_done[bsel])
        stream.wait_event(d2h_done[bsel])  # dC[bsel] has been read back
        B.check(h.set_epilogue(bias=dbias[bsel], bias_type=Nn.GRX_R_32F), "set_epilogue")
        s = h.gemm_ex(Nn.OP_T, Nn.OP_N, M, nl, K, 1.0, dA[bsel], Nn.GRX_R_16BF, K, dB[bsel], Nn.GRX_R_16BF, K, 0.0,
                      dC[bsel], Nn.GRX_R_16BF, M)
        if s != Nn.SUCCESS:
            raise RuntimeError(Nn.STATUS[s])
        gemm_done[bsel].record(stream)
        with torch.cuda.stream(down):
            down.wait_event(gemm_done[bsel])
            hC[bsel].copy_(dC[bsel], non_blocking=True)
            d2h_done[bsel].record(down)

    e2e_steps = max(4, min(args.steps, 12))
    for i in range(2):
        e2e_step(i)
    torch.cuda.synchronize()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(up)
    for i in range(e2e_steps):
        e2e_step(i)
    stream.wait_event(d2h_done[(e2e_steps - 1) & 1])
    stream.wait_event(d2h_done[(e2e_steps - 2) & 1])
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1) / e2e_steps)
    h2d = (hA.numel() + Bl.numel()) * 2 + bias.numel() * 4
    d2h = C.numel() * 2
    e2e = {"value": flops_total / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s", "h2d_bytes_per_step": h2d * world,
           "d2h_bytes_per_step": d2h * world, "ms_per_step": e2e_ms,
           "note": "every step: H2D from pinned memory of this rank's 1/N row band of A (then one NCCL "
                   "all-gather of A over NVLink), its B columns and bias; GemmEx through the C-ABI; D2H of its C "
                   "columns; steps pipelined over two copy streams (uploads of step i+1 overlap the GEMM and "
                   "download of step i)"}
    del hA, hB, hC, dA, dB, dbias, dC
    h.clear_epilogue()

    attention = run_attention_sharded(args, peaks, dev, stream, rank, world, barrier, max_over_ranks)

    secondary = {}
    cpu = None
    if rank == 0:
        if not args.no_secondary:
            del A, Bl, C
            torch.cuda.empty_cache()
            secondary = run_secondary(args, peaks, dev, stream)
        threads = len(os.sched_getaffinity(0))
        v, cols, dt = cpu_gemm_sample(args.cpu_seconds, threads)
        cpu = {"value": v, "unit": "TFLOP/s", "cores": threads, "kind": "port",
               "sample": f"{cols} of {N} output columns of the 8192^3 GEMM ({dt:.1f} s, fp64 naive loop, oracle "
                         "restatement of tests/libs/test_grxblas.cpp:63-80)"}
    if rank == 0:
        line = {
            "metric": "GEMM TFLOP/s (% dense tensor peak) at 1/2/4/8 B200; attention TFLOP/s; norm GB/s",
            "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps, "warmup": max(args.warmup, 3),
            "ms_per_step": ms, "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic: A, B ~N(0,1)/sqrt(K) bf16, bias ~N(0,0.02) fp32, seeded",
            "config": config_dict(world),
            "frac_of_peak": value / (peak * world),
            "roofline": roofline, "clocks": clk, "e2e": e2e, "gpu_launches": args.steps,
            "attention": attention,
            "cpu_baseline": cpu, "secondary": secondary,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()
    return 0


def run_attention_sharded(args, peaks, dev, stream, rank, world, barrier, max_over_ranks):
    """BASELINE config 4 (causal attention forward, bf16, B=8 H=32 S=4096 D=128,
    fp32 LSE) sharded over batch x heads: every rank runs grxdnnAttentionForward
    on its 256 / world (batch, head) pairs through shard.attention_head_parallel,
    with no collective (each rank keeps its own heads). Device time per step is
    the max over ranks; value = the whole job's FLOP / that time."""
    import torch

    from grxcp_b200 import dnn as D
    from grxcp_b200 import shard

    Bq, H, S, Dh = 8, 32, 4096, 128
    g = torch.Generator(device=dev).manual_seed(99)
    q = torch.randn(Bq, H, S, Dh, device=dev, generator=g).to(torch.bfloat16)
    k = torch.randn(Bq, H, S, Dh, device=dev, generator=g).to(torch.bfloat16)
    v = torch.randn(Bq, H, S, Dh, device=dev, generator=g).to(torch.bfloat16)
    o = torch.empty_like(q)
    lse = torch.empty(Bq, H, S, device=dev)
    dh = D.Handle()
    dh.set_stream(stream)

    def step():
        st = shard.attention_head_parallel(dh, q, k, v, o, 1 / math.sqrt(Dh), True, lse, rank=rank, world=world)
        if st != 0:
            raise RuntimeError(f"grxdnnAttentionForward status {st}")

    steps = max(3, min(args.steps, 10))
    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(steps):
        step()
    b.record(stream)
    torch.cuda.synchronize()
    ms = max_over_ranks(a.elapsed_time(b) / steps)
    barrier()
    st = dh.execution_status()
    dh.close()
    if st != 0:
        raise RuntimeError(f"attention kernel reported status {st}")
    fl = 2.0 * Bq * H * S * S * Dh  # causal: half of 4 * B * H * S^2 * D
    peak = peaks["bf16_tflops"]
    del q, k, v, o, lse
    torch.cuda.empty_cache()
    return {"value": fl / ms / 1e9, "unit": "TFLOP/s", "ms": ms, "n_gpus": world, "steps": steps,
            "frac": fl / ms / 1e9 / (peak * world), "scaling": "strong",
            "config": f"causal, bf16, B=8 H=32 S=4096 D=128, fp32 LSE; {Bq * H // world} (batch, head) pairs per "
                      "rank, no collective; FLOP = 2*B*H*S^2*D; max over ranks"}


def measure_8bit_peaks(dev, stream):
    """Roofline denominators for the 8-bit kinds, measured on this GPU the way
    the bf16 peak is: a vendor-library dense GEMM at 8192^3, timed with CUDA
    events (e4m3 via torch._scaled_mm, int8 via torch._int_mm). Returns
    (fp8 TFLOP/s, int8 TOP/s)."""
    import torch

    n = 8192
    g = torch.Generator(device=dev).manual_seed(5)
    a = torch.randn(n, n, device=dev, generator=g).div(8).to(torch.float8_e4m3fn)
    b = torch.randn(n, n, device=dev, generator=g).div(8).to(torch.float8_e4m3fn).t()  # column-major
    one = torch.ones((), device=dev)
    ms8 = _time(lambda: torch._scaled_mm(a, b, scale_a=one, scale_b=one, out_dtype=torch.bfloat16), 10, stream)
    ia = torch.randint(-128, 128, (n, n), device=dev, dtype=torch.int8, generator=g)
    ib = torch.randint(-128, 128, (n, n), device=dev, dtype=torch.int8, generator=g).t()
    msi = _time(lambda: torch._int_mm(ia, ib), 10, stream)
    del a, b, ia, ib
    torch.cuda.empty_cache()
    fl = 2.0 * n ** 3
    return fl / ms8 / 1e9, fl / msi / 1e9


def _quantize_e4m3(x):
    """[batch, rows, k] fp32 -> e4m3 codes and one scale (amax / 448) per batch member."""
    import torch

    scale = (x.abs().amax(dim=(1, 2)) / 448.0).clamp_min(1e-30)
    return (x / scale[:, None, None]).to(torch.float8_e4m3fn), scale


def _quantize_i8_rows(x):
    """[batch, rows, k] fp32 -> int8 codes and one scale (amax / 127) per row, shared by the batch."""
    import torch

    scale = (x.abs().amax(dim=(0, 2)) / 127.0).clamp_min(1e-30)
    return torch.clamp(torch.round(x / scale[None, :, None]), -127, 127).to(torch.int8), scale


def _time(fn, iters, stream):
    import torch

    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(iters):
        fn()
    b.record(stream)
    torch.cuda.synchronize()
    return a.elapsed_time(b) / iters


def _time_graph(fn, iters, handle, stream):
    """Per-call device time of a launch-bound call: `iters` calls captured in
    one CUDA graph on a side stream (the handle's stream during capture), then
    the graph replayed between CUDA events. The eager loop of these calls is
    bound by the host's per-call cost (ctypes, tensor-map encoding)."""
    import torch

    side = torch.cuda.Stream()
    handle.set_stream(side)
    try:
        with torch.cuda.stream(side):
            for _ in range(3):
                fn()
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=side):
            for _ in range(iters):
                fn()
        g.replay()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(side):
            a.record(side)
            g.replay()
            b.record(side)
        torch.cuda.synchronize()
        return a.elapsed_time(b) / iters
    finally:
        handle.set_stream(stream)


def run_secondary(args, peaks, dev, stream):
    """The other BASELINE configs on rank 0, each timed with CUDA events (inputs larger than L2)."""
    import torch

    from grxcp_b200 import _native as Nn
    from grxcp_b200 import blas as B
    from grxcp_b200 import dnn as D

    out = {}
    dh = D.Handle()
    dh.set_stream(stream)
    bh = B.Handle()
    bh.set_stream(stream)
    g = torch.Generator(device=dev).manual_seed(7)
    hbm = peaks["hbm_gbs"]
    bf16_peak = peaks["bf16_tflops"]

    # config 3: RMSNorm / LayerNorm [65536, 8192] bf16
    x = torch.randn(65536, 8192, device=dev, generator=g).to(torch.bfloat16)
    y = torch.empty_like(x)
    gamma = 1 + 0.02 * torch.randn(8192, device=dev, generator=g)
    beta = 0.02 * torch.randn(8192, device=dev, generator=g)
    nbytes = 2 * x.numel() * 2 + 8192 * 4
    ms = _time(lambda: dh.rmsnorm(x, gamma, 1e-5, y), 20, stream)
    out["rmsnorm"] = {"value": nbytes / ms / 1e6, "unit": "GB/s", "ms": ms, "frac": nbytes / ms / 1e6 / hbm,
                      "config": "bf16 [65536, 8192], fp32 gamma, eps 1e-5"}
    ms = _time(lambda: dh.layernorm(x, gamma, beta, 1e-5, y), 20, stream)
    nb = nbytes + 8192 * 4
    out["layernorm"] = {"value": nb / ms / 1e6, "unit": "GB/s", "ms": ms, "frac": nb / ms / 1e6 / hbm,
                        "config": "bf16 [65536, 8192], fp32 gamma/beta, eps 1e-5"}
    # softmax over rows and GELU on the same bf16 tensor: read once, written once
    ms = _time(lambda: dh.softmax(x, y), 20, stream)
    out["softmax"] = {"value": (nbytes - 8192 * 4) / ms / 1e6, "unit": "GB/s", "ms": ms,
                      "frac": (nbytes - 8192 * 4) / ms / 1e6 / hbm, "config": "bf16 [65536, 8192], fp32 math"}
    ms = _time(lambda: dh.gelu(x, y, 0), 20, stream)
    out["gelu"] = {"value": (nbytes - 8192 * 4) / ms / 1e6, "unit": "GB/s", "ms": ms,
                   "frac": (nbytes - 8192 * 4) / ms / 1e6 / hbm, "config": "bf16, 2^29 elements, erf form"}
    # their backward passes: two tensors read, one written
    dy0 = torch.randn(65536, 8192, device=dev, generator=g).to(torch.bfloat16)
    nb3 = 3 * x.numel() * 2
    ms = _time(lambda: dh.softmax_backward(y, dy0, y), 20, stream)
    out["softmax_backward"] = {"value": nb3 / ms / 1e6, "unit": "GB/s", "ms": ms, "frac": nb3 / ms / 1e6 / hbm,
                               "config": "bf16 [65536, 8192], dx written over y"}
    ms = _time(lambda: dh.gelu_backward(x, dy0, y, 0), 20, stream)
    out["gelu_backward"] = {"value": nb3 / ms / 1e6, "unit": "GB/s", "ms": ms, "frac": nb3 / ms / 1e6 / hbm,
                            "config": "bf16, 2^29 elements, erf form"}
    del dy0
    # norm backward on the same shape: x and dy read, dx written (saved statistics)
    dy = torch.randn(65536, 8192, device=dev, generator=g).to(torch.bfloat16)
    mean = torch.empty(65536, device=dev)
    rstd = torch.empty(65536, device=dev)
    dgamma = torch.empty(8192, device=dev)
    dbeta = torch.empty(8192, device=dev)
    D.check(dh.layernorm(x, gamma, beta, 1e-5, y, mean, rstd))
    nbw = 3 * x.numel() * 2
    ms = _time(lambda: dh.rmsnorm_backward(dy, x, gamma, 1e-5, y, rstd, dgamma), 20, stream)
    out["rmsnorm_backward"] = {"value": nbw / ms / 1e6, "unit": "GB/s", "ms": ms, "frac": nbw / ms / 1e6 / hbm,
                               "config": "bf16 [65536, 8192], saved rstd, dx + fp32 dgamma"}
    ms = _time(lambda: dh.layernorm_backward(dy, x, gamma, 1e-5, y, mean, rstd, dgamma, dbeta), 20, stream)
    out["layernorm_backward"] = {"value": nbw / ms / 1e6, "unit": "GB/s", "ms": ms, "frac": nbw / ms / 1e6 / hbm,
                                 "config": "bf16 [65536, 8192], saved mean/rstd, dx + fp32 dgamma/dbeta"}
    del x, y, dy
    torch.cuda.empty_cache()

    # config 4: causal attention B=8 H=32 S=4096 D=128
    q = torch.randn(8, 32, 4096, 128, device=dev, generator=g).to(torch.bfloat16)
    k = torch.randn_like(q)
    v = torch.randn_like(q)
    o = torch.empty_like(q)
    lse = torch.empty(8, 32, 4096, device=dev)
    fl = 2.0 * 8 * 32 * 4096 * 4096 * 128
    ms = _time(lambda: dh.attention(q, k, v, o, 1 / math.sqrt(128), True, lse), 10, stream)
    out["attention"] = {"value": fl / ms / 1e9, "unit": "TFLOP/s", "ms": ms, "frac": fl / ms / 1e9 / bf16_peak,
                        "config": "causal, bf16, B=8 H=32 S=4096 D=128, fp32 LSE; FLOP = 2*B*H*S^2*D"}
    # backward of the same call (dQ, dK, dV from O, LSE and a random dO)
    dout = torch.randn_like(q)
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    ms = _time(lambda: dh.attention_backward(q, k, v, o, dout, lse, 1 / math.sqrt(128), True, dq, dk, dv), 5, stream)
    out["attention_backward"] = {
        "value": 2.5 * fl / ms / 1e9, "unit": "TFLOP/s", "ms": ms, "frac": 2.5 * fl / ms / 1e9 / bf16_peak,
        "config": "causal, bf16, B=8 H=32 S=4096 D=128; FLOP = 2.5 x forward (five GEMMs); the kernels execute "
                  "seven (S and dP are recomputed by the dQ pass instead of fp32 atomics)"}
    del q, k, v, o, lse, dout, dq, dk, dv
    torch.cuda.empty_cache()

    # config 5: fp8 e4m3 strided-batched MLP GEMM, batch 16, 4096 x 14336 x 4096, per-tensor scales, bf16 out
    bt, m5, n5, k5 = 16, 4096, 14336, 4096
    # A/B ~ N(0,1) quantised to e4m3 with per-tensor (per batch member) scales amax / 448
    a8, sa = _quantize_e4m3(torch.randn(bt, m5, k5, device=dev, generator=g))
    b8, sb = _quantize_e4m3(torch.randn(bt, n5, k5, device=dev, generator=g))
    c5 = torch.empty(bt, n5, m5, device=dev, dtype=torch.bfloat16)
    bh.set_epilogue(scale_mode=Nn.SCALE_TENSOR, scale_a=sa, scale_b=sb, stride_scale_a=1, stride_scale_b=1)
    fl5 = 2.0 * bt * m5 * n5 * k5
    ms = _time(lambda: bh.gemm_strided_batched_ex(Nn.OP_T, Nn.OP_N, m5, n5, k5, 1.0, a8, Nn.GRX_R_8F_E4M3, k5,
                                                  m5 * k5, b8, Nn.GRX_R_8F_E4M3, k5, n5 * k5, 0.0, c5,
                                                  Nn.GRX_R_16BF, m5, m5 * n5, bt), 5, stream)
    fp8_peak, i8_peak = measure_8bit_peaks(dev, stream)
    out["fp8_batched_gemm"] = {"value": fl5 / ms / 1e9, "unit": "TFLOP/s", "ms": ms,
                               "frac": fl5 / ms / 1e9 / fp8_peak, "peak": fp8_peak,
                               "peak_note": "measured here: cuBLASLt e4m3 GEMM 8192^3 (torch._scaled_mm), burst",
                               "config": "e4m3, batch 16, 4096x14336x4096, per-tensor scales, bf16 out"}
    # int8 variant with per-row / per-column scales
    # int8 codes with per-row (A) / per-column (B) scales amax / 127
    i8a, sra = _quantize_i8_rows(torch.randn(bt, m5, k5, device=dev, generator=g))
    i8b, srb = _quantize_i8_rows(torch.randn(bt, n5, k5, device=dev, generator=g))
    bh.set_epilogue(scale_mode=Nn.SCALE_ROWCOL, scale_a=sra, scale_b=srb)
    ms = _time(lambda: bh.gemm_strided_batched_ex(Nn.OP_T, Nn.OP_N, m5, n5, k5, 1.0, i8a, Nn.GRX_R_8I, k5,
                                                  m5 * k5, i8b, Nn.GRX_R_8I, k5, n5 * k5, 0.0, c5,
                                                  Nn.GRX_R_16BF, m5, m5 * n5, bt), 5, stream)
    out["int8_rowcol_batched_gemm"] = {"value": fl5 / ms / 1e9, "unit": "TOP/s", "ms": ms,
                                       "frac": fl5 / ms / 1e9 / i8_peak, "peak": i8_peak,
                                       "peak_note": "measured here: cuBLASLt int8 GEMM 8192^3 -> int32 "
                                                    "(torch._int_mm), burst",
                                       "config": "int8, batch 16, 4096x14336x4096, per-row/col scales, bf16 out"}
    bh.clear_epilogue()
    del a8, b8, i8a, i8b, c5
    torch.cuda.empty_cache()

    # NHWC pooling (3x3, stride 2, pad 1, max) over a ResNet-style bf16 activation
    xp = torch.randn(128, 56, 56, 256, device=dev, generator=g).to(torch.bfloat16)
    yp = torch.empty(128, 28, 28, 256, device=dev, dtype=torch.bfloat16)
    npb = (xp.numel() + yp.numel()) * 2
    ms = _time(lambda: dh.pool2d(xp, yp, (3, 3), (1, 1), (2, 2), 0), 20, stream)
    out["pool2d"] = {"value": npb / ms / 1e6, "unit": "GB/s", "ms": ms, "frac": npb / ms / 1e6 / hbm,
                     "config": "bf16 NHWC [128, 56, 56, 256], 3x3 max, stride 2, pad 1; input read once + output"}
    del xp, yp
    # config 1: fp32 SGEMM 512^3 and int8 512^3
    a = torch.rand(512 * 512, device=dev, generator=g) * 2 - 1
    b = torch.rand(512 * 512, device=dev, generator=g) * 2 - 1
    c = torch.empty(512 * 512, device=dev)
    sg = lambda: bh.sgemm(0, 0, 512, 512, 512, 1.0, b, 512, a, 512, 0.0, c, 512)  # noqa: E731
    ms_eager = _time(sg, 50, stream)
    ms = _time_graph(sg, 50, bh, stream)
    out["sgemm_512"] = {"value": 2 * 512 ** 3 / ms / 1e9, "unit": "TFLOP/s", "ms": ms, "ms_eager": ms_eager,
                        "config": "fp32 row-major 512^3 via swapped column-major call; ms = device time per call "
                                  "(CUDA graph of 50 calls), ms_eager = eager back-to-back calls (host-bound)"}
    ia = torch.randint(-128, 128, (512 * 512,), device=dev, dtype=torch.int8)
    ic = torch.empty(512 * 512, device=dev, dtype=torch.int32)
    i8 = lambda: bh.gemm_ex(0, 0, 512, 512, 512, 1.0, ia, Nn.GRX_R_8I, 512, ia, Nn.GRX_R_8I, 512, 0.0, ic,  # noqa: E731
                            Nn.GRX_R_32I, 512)
    ms_eager = _time(i8, 50, stream)
    ms = _time_graph(i8, 50, bh, stream)
    out["int8_512"] = {"value": 2 * 512 ** 3 / ms / 1e9, "unit": "TOP/s", "ms": ms, "ms_eager": ms_eager,
                       "config": "int8 512^3 -> int32, bit-exact path; ms = device time per call (CUDA graph of "
                                 "50 calls), ms_eager = eager back-to-back calls (host-bound)"}
    if dh.execution_status() != Nn.SUCCESS or bh.execution_status() != Nn.SUCCESS:
        out["error"] = "a kernel reported a bounded-wait timeout"
    return out


def run_profile(args):
    """One workload, warmup + steps launches, nothing else: the command ncu captures."""
    import torch

    from grxcp_b200 import _native as Nn
    from grxcp_b200 import blas as B
    from grxcp_b200 import dnn as D

    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(1)
    n_iter = args.warmup + args.steps
    if args.profile == "config1":
        # BASELINE config 1 (512^3): int8 and bf16 GemmEx with the narrow tiles, then with
        # 128 x 256 tiles (GRX_GEMM_WIDE_TILES), then SGEMM with 4 k-groups and with one.
        h = B.Handle()
        ia = torch.randint(-128, 128, (512 * 512,), dtype=torch.int8, device=dev, generator=g)
        ic = torch.empty(512 * 512, dtype=torch.int32, device=dev)
        ba = torch.randn(512 * 512, device=dev, generator=g).to(torch.bfloat16)
        bc = torch.empty(512 * 512, device=dev, dtype=torch.bfloat16)
        fa = torch.rand(512 * 512, device=dev, generator=g) * 2 - 1
        fc = torch.empty(512 * 512, device=dev)
        for env in (None, "GRX_GEMM_WIDE_TILES"):
            if env:
                os.environ[env] = "1"
            for _ in range(n_iter):
                B.check(h.gemm_ex(0, 0, 512, 512, 512, 1.0, ia, Nn.GRX_R_8I, 512, ia, Nn.GRX_R_8I, 512, 0.0, ic,
                                  Nn.GRX_R_32I, 512))
            for _ in range(n_iter):
                B.check(h.gemm_ex(1, 0, 512, 512, 512, 1.0, ba, Nn.GRX_R_16BF, 512, ba, Nn.GRX_R_16BF, 512, 0.0, bc,
                                  Nn.GRX_R_16BF, 512))
            os.environ.pop("GRX_GEMM_WIDE_TILES", None)
        for env in (None, "GRX_SGEMM_KG1"):
            if env:
                os.environ[env] = "1"
            for _ in range(n_iter):
                B.check(h.sgemm(0, 0, 512, 512, 512, 1.0, fa, 512, fa, 512, 0.0, fc, 512))
            os.environ.pop("GRX_SGEMM_KG1", None)
        torch.cuda.synchronize()
        B.check(h.execution_status())
        h.close()
        return
    if args.profile in ("gemm", "fp8"):
        h = B.Handle()
        if args.profile == "gemm":
            A = (torch.randn(M, K, device=dev, generator=g) / math.sqrt(K)).to(torch.bfloat16)
            nc = args.profile_cols or N  # one rank's column slice of the N-GPU run (N / world)
            Bm = (torch.randn(nc, K, device=dev, generator=g) / math.sqrt(K)).to(torch.bfloat16)
            C = torch.empty(nc, M, device=dev, dtype=torch.bfloat16)
            bias = torch.randn(nc, device=dev, generator=g) * 0.02
            h.set_epilogue(bias=bias, bias_type=Nn.GRX_R_32F)
            for _ in range(n_iter):
                B.check(h.gemm_ex(1, 0, M, nc, K, 1.0, A, Nn.GRX_R_16BF, K, Bm, Nn.GRX_R_16BF, K, 0.0, C,
                                  Nn.GRX_R_16BF, M))
        else:
            bt, m5, n5, k5 = 16, 4096, 14336, 4096
            a8, sa = _quantize_e4m3(torch.randn(bt, m5, k5, device=dev, generator=g))
            b8, sb = _quantize_e4m3(torch.randn(bt, n5, k5, device=dev, generator=g))
            c5 = torch.empty(bt, n5, m5, device=dev, dtype=torch.bfloat16)
            h.set_epilogue(scale_mode=Nn.SCALE_TENSOR, scale_a=sa, scale_b=sb, stride_scale_a=1, stride_scale_b=1)
            for _ in range(n_iter):
                B.check(h.gemm_strided_batched_ex(1, 0, m5, n5, k5, 1.0, a8, Nn.GRX_R_8F_E4M3, k5, m5 * k5, b8,
                                                  Nn.GRX_R_8F_E4M3, k5, n5 * k5, 0.0, c5, Nn.GRX_R_16BF, m5,
                                                  m5 * n5, bt))
        torch.cuda.synchronize()
        B.check(h.execution_status())
    else:
        dh = D.Handle()
        if args.profile == "attention":
            q = torch.randn(8, 32, 4096, 128, device=dev, generator=g).to(torch.bfloat16)
            k, v, o = torch.randn_like(q), torch.randn_like(q), torch.empty_like(q)
            lse = torch.empty(8, 32, 4096, device=dev)
            for _ in range(n_iter):
                D.check(dh.attention(q, k, v, o, 1 / math.sqrt(128), True, lse))
        elif args.profile == "attention_bwd":
            # config 4 per head at batch 2 (a quarter of the heads), so a capture holds ~0.5 GB
            q = torch.randn(2, 32, 4096, 128, device=dev, generator=g).to(torch.bfloat16)
            k, v, o, do = torch.randn_like(q), torch.randn_like(q), torch.empty_like(q), torch.randn_like(q)
            dq, dk, dv = torch.empty_like(q), torch.empty_like(q), torch.empty_like(q)
            lse = torch.empty(2, 32, 4096, device=dev)
            D.check(dh.attention(q, k, v, o, 1 / math.sqrt(128), True, lse))
            for _ in range(n_iter):
                D.check(dh.attention_backward(q, k, v, o, do, lse, 1 / math.sqrt(128), True, dq, dk, dv))
        elif args.profile in ("rmsnorm_bwd", "layernorm_bwd"):
            x = torch.randn(16384, 8192, device=dev, generator=g).to(torch.bfloat16)
            dy, dx = torch.randn_like(x), torch.empty_like(x)
            gamma, beta = torch.ones(8192, device=dev), torch.zeros(8192, device=dev)
            mean, rstd = torch.empty(16384, device=dev), torch.empty(16384, device=dev)
            dgamma, dbeta = torch.empty(8192, device=dev), torch.empty(8192, device=dev)
            D.check(dh.layernorm(x, gamma, beta, 1e-5, dx, mean, rstd))
            for _ in range(n_iter):
                if args.profile == "rmsnorm_bwd":
                    D.check(dh.rmsnorm_backward(dy, x, gamma, 1e-5, dx, rstd, dgamma))
                else:
                    D.check(dh.layernorm_backward(dy, x, gamma, 1e-5, dx, mean, rstd, dgamma, dbeta))
        elif args.profile == "conv":
            x = torch.randn(128, 28, 28, 128, device=dev, generator=g).to(torch.bfloat16)
            w = (torch.randn(128, 3, 3, 128, device=dev, generator=g) / 34).to(torch.bfloat16)
            y = torch.empty(128, 28, 28, 128, device=dev).to(torch.bfloat16)
            for _ in range(n_iter):
                D.check(dh.conv2d(x, w, y, (1, 1)))
        else:
            x = torch.randn(65536, 8192, device=dev, generator=g).to(torch.bfloat16)
            y = torch.empty_like(x)
            gamma = torch.ones(8192, device=dev)
            beta = torch.zeros(8192, device=dev)
            for _ in range(n_iter):
                if args.profile == "rmsnorm":
                    D.check(dh.rmsnorm(x, gamma, 1e-5, y))
                else:
                    D.check(dh.layernorm(x, gamma, beta, 1e-5, y))
        torch.cuda.synchronize()
        D.check(dh.execution_status())
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="grxcp", choices=["grxcp", "reference"])
    ap.add_argument("--no-secondary", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=20.0)
    ap.add_argument("--profile-cols", type=int, default=0,
                    help="--profile gemm: columns of the slice (a rank's N / world); default N")
    ap.add_argument("--profile", choices=["gemm", "attention", "rmsnorm", "layernorm", "fp8", "attention_bwd",
                                          "rmsnorm_bwd", "layernorm_bwd", "conv", "config1"],
                    help="run only this kernel warmup+steps times (for ncu captures); prints no JSON")
    args = ap.parse_args()
    if args.impl == "reference":
        return run_reference(args)
    if args.profile:
        return run_profile(args)
    return run_gpu(args)


if __name__ == "__main__":
    sys.exit(main())
