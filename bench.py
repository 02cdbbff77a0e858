#!/usr/bin/env python
"""Benchmark of breccia's hot path on B200: cast + scaled GEMM.

Headline workload (Float8CurrentScaling E4M3):
  A bf16 (16384, 8192) ~ N(0,1) with 0.1% of entries replaced by N(0,1)*50,
  W bf16 (8192, 8192) ~ N(0,0.02), held as W^T (N, K) (nn.Linear orientation).
  One step = per-tensor cast of A + per-tensor cast of W^T + the 16384 x 8192 x
  8192 tcgen05 FP8 GEMM -> bf16.
  N GPUs, default (--shard batch, data parallel, "weak" scaling): every rank
  holds its own batch of 16384 activation rows (rank 0's is the C2 A above,
  the others are seeded per rank) and the whole weight. The activations'
  per-tensor scale is that of the concatenated global batch (16384*N rows):
  one NCCL all-reduce(MAX) of a 4-byte amax word, overlapped with the
  weight's cast. Per-GPU work is fixed as N grows.
  --shard weight ("strong" scaling): W^T is split along N (rows); the
  weight's amax is reduced with one all-reduce; A is replicated; each rank
  computes its C[:, shard]. Total work is fixed.

value = total 2*M*N*K over all ranks / step time (max over ranks).
e2e   = the same through the public API with the inputs copied from pinned
        host memory and the output C copied back inside every step.

Usage: python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]
Under torchrun one process per GPU; rank 0 prints one JSON line.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

M, N, K = 16384, 8192, 8192
FLOPS = 2.0 * M * N * K
WORKLOAD = ("C2 Float8CurrentScaling E4M3 per-tensor: A bf16 (16384, 8192) N(0,1) with 0.1% "
            "N(0,1)*50 outliers, W bf16 (8192, 8192) N(0,0.02) held as W^T; cast A + cast W "
            "+ 16384x8192x8192 tcgen05 FP8 GEMM -> bf16")
METRIC = "scaled-matmul TFLOP/s (C2 per-tensor FP8: cast A + cast W + GEMM, whole job)"

# DRAM bytes (read + write) of one launch of the GEMM kernel on this
# workload, from one ncu capture of `bench.py --steps 1 --warmup 3 --no-e2e
# --no-cpu-baseline` (dram__bytes_read.sum 679.50 MB + dram__bytes_write.sum
# 248.64 MB; profiles/gemm_fp8_pertensor_c2.md).
GEMM_DRAM_BYTES = 679.50e6 + 248.64e6


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--shard", default="batch", choices=["batch", "weight"],
                    help="N>1 layout: per-rank activation batches with the weight replicated "
                         "(weak scaling, default) or the weight split along N (strong)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--per-recipe", action="store_true",
                    help="also measure every BASELINE config's cast GB/s and GEMM TFLOP/s")
    ap.add_argument("--cpu-rows", type=int, default=None,
                    help="rows of A / W^T the CPU port encodes per sample (default 64 for "
                         "cpu_baseline, 16 per step for --impl reference)")
    ap.add_argument("--ncu-case", default=None, choices=sorted(NCU_CASES),
                    help="run one kernel on a small case (inputs > L2, < 1 GB) 3 times, for ncu")
    return ap.parse_args()


# --------------------------------------------------------------- CPU side


def _cpu_encode_rows(args):
    """Worker: the reference's per-tensor encode (literal LUT search) of rows."""
    x, scale, fmt = args
    import numpy as np
    from oracle import codec
    x = np.asarray(x, dtype=np.float32)
    enc = codec.encode_e4m3 if fmt == "E4M3" else codec.encode_e5m2
    t0 = time.perf_counter()
    enc(x / np.float32(scale), literal=True)
    return time.perf_counter() - t0


def cpu_reference_step(A_np, Wt_np, rows, pool, nproc):
    """Time the reference NumPy path on a bounded sample of the C2 step and
    extrapolate to the whole step by rows (the per-tensor encode is elementwise
    once the scale is known; the matmul is row-separable in A).

    Returns (seconds for the whole step, breakdown dict)."""
    import numpy as np
    from oracle import codec, cast as ocast

    t = {}
    t0 = time.perf_counter()
    amax_a = codec.tensor_amax(A_np)
    t["amax_A"] = time.perf_counter() - t0
    t0 = time.perf_counter()
    amax_w = codec.tensor_amax(Wt_np)
    t["amax_W"] = time.perf_counter() - t0
    sa = np.float32(amax_a / 448.0)
    sw = np.float32(amax_w / 448.0)
    # encode `rows` rows of A and of W^T, split over the pool
    chunks = [(A_np[i::nproc][: max(1, rows // nproc)], sa, "E4M3") for i in range(nproc)]
    chunks += [(Wt_np[i::nproc][: max(1, rows // nproc)], sw, "E4M3") for i in range(nproc)]
    t0 = time.perf_counter()
    list(pool.map(_cpu_encode_rows, chunks))
    t_enc = time.perf_counter() - t0  # wall time for ~rows rows of A and of W^T
    per_row_enc = t_enc / (2 * nproc * max(1, rows // nproc))
    t["encode_A"] = per_row_enc * A_np.shape[0]
    t["encode_W"] = per_row_enc * Wt_np.shape[0]
    # reference matmul: dequantize both (LUT decode * scale), float32 sgemm
    qa = codec.encode_e4m3(A_np[:rows] / sa)
    qw_rows = codec.encode_e4m3(Wt_np[:rows] / sw)
    t0 = time.perf_counter()
    da = codec.decode_e4m3(qa) * sa
    t["dequant_A"] = (time.perf_counter() - t0) * A_np.shape[0] / rows
    t0 = time.perf_counter()
    dw = codec.decode_e4m3(qw_rows) * sw
    t["dequant_W"] = (time.perf_counter() - t0) * Wt_np.shape[0] / rows
    dW = np.ascontiguousarray(np.broadcast_to(dw[:1], Wt_np.shape)).T  # full-size operand
    t0 = time.perf_counter()
    _ = da @ dW
    t["sgemm"] = (time.perf_counter() - t0) * A_np.shape[0] / rows
    return sum(t.values()), t


def run_reference(args):
    """--impl reference: the oracle port of breccia's NumPy path on the host.
    Each step is a bounded sample (16 rows of A and of W^T encoded, about a
    second of host time) extrapolated to the whole C2 step, so the run stays
    within minutes for any --steps / --warmup the driver passes."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    if args.cpu_rows is None:
        args.cpu_rows = 16
    import multiprocessing as mp
    import numpy as np
    from concurrent.futures import ProcessPoolExecutor
    A_np, Wt_np = host_inputs_numpy()
    nproc = os.cpu_count() or 1
    times = []
    with ProcessPoolExecutor(max_workers=nproc, mp_context=mp.get_context("spawn")) as pool:
        _warm_pool(pool, nproc)
        for i in range(args.warmup + args.steps):
            t, _ = cpu_reference_step(A_np, Wt_np, args.cpu_rows, pool, nproc)
            if i >= args.warmup:
                times.append(t)
    sec = statistics.mean(times)
    value = FLOPS / sec / 1e12
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "TFLOP/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": sec * 1e3, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32 (numpy)", "data": "synthetic",
        "config": {"workload": WORKLOAD, "M": M, "N": N, "K": K},
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": nproc, "kind": "port",
                         "sample": f"{args.cpu_rows} rows of A and of W^T encoded per step "
                                   "(literal LUT search, process pool), full-tensor amax, "
                                   f"{args.cpu_rows}-row dequant + sgemm; extrapolated by rows"},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def host_inputs_numpy():
    """C2 inputs as float32 NumPy arrays (the reference's np.asarray(x, float32)
    of the bf16 values), generated with the same seeded torch generator."""
    A, Wt = make_inputs("cpu")
    return A.float().numpy(), Wt.float().numpy()


# --------------------------------------------------------------- GPU side


def _make_a(g, device):
    import torch
    A = torch.randn(M, K, generator=g, device=device)
    mask = torch.rand(M, K, generator=g, device=device) < 0.001
    A = torch.where(mask, torch.randn(M, K, generator=g, device=device) * 50, A)
    return A.to(torch.bfloat16)


def make_inputs(device, batch_seed=None):
    """C2's A and W^T (seed 0). With ``batch_seed`` the returned A is instead
    a fresh batch of the same distribution from that seed (W^T unchanged)."""
    import torch
    g = torch.Generator(device=device).manual_seed(0)
    A = _make_a(g, device)
    W = (torch.randn(K, N, generator=g, device=device) * 0.02).to(torch.bfloat16)
    if batch_seed is not None:
        del A
        A = _make_a(torch.Generator(device=device).manual_seed(batch_seed), device)
    return A, W.t().contiguous()


class Clocks:
    """SM clock and throttle reasons sampled every 5 ms through NVML (the
    source nvidia-smi reads) while the timed region runs; nvidia-smi's own
    200 ms loop is too coarse for a region of a few tens of milliseconds."""

    REASONS = {"hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "sw_thermal_slowdown": 0x20,
               "sw_power_cap": 0x4, "hw_power_brake_slowdown": 0x80}

    def __init__(self, uuid):
        self.uuid = uuid
        self.samples = []
        self._stop = None
        self._thread = None

    def __enter__(self):
        import threading
        try:
            import pynvml
            pynvml.nvmlInit()
            handle = None
            for i in range(pynvml.nvmlDeviceGetCount()):
                h = pynvml.nvmlDeviceGetHandleByIndex(i)
                u = pynvml.nvmlDeviceGetUUID(h)
                u = u.decode() if isinstance(u, bytes) else u
                if self.uuid is None or u == self.uuid:
                    handle = h
                    break
            if handle is None:
                return self
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(handle, pynvml.NVML_CLOCK_SM)
        except Exception:  # no NVML: report no samples
            return self
        self._stop = threading.Event()

        def run():
            while not self._stop.is_set():
                try:
                    mhz = pynvml.nvmlDeviceGetClockInfo(handle, pynvml.NVML_CLOCK_SM)
                    rs = pynvml.nvmlDeviceGetCurrentClocksEventReasons(handle)
                    self.samples.append((mhz, rs))
                except Exception:
                    pass
                self._stop.wait(0.005)

        self._thread = threading.Thread(target=run, daemon=True)
        self._thread.start()
        return self

    def __exit__(self, *exc):
        if self._thread is not None:
            self._stop.set()
            self._thread.join(timeout=2)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0,
                    "source": "nvml"}
        active = sorted({n for _, rs in self.samples for n, bit in self.REASONS.items()
                         if rs & bit})
        return {"sm_mhz": statistics.median(m for m, _ in self.samples),
                "sm_max_mhz": getattr(self, "max_mhz", None), "reasons": active,
                "samples": len(self.samples), "source": "nvml, 5 ms period"}


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return json.load(f), "measured"
    except OSError:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, \
            "fallback"


def run_ours(args):
    import torch
    import torch.distributed as dist
    import breccia_b200 as bb
    from breccia_b200.dist import shard_rows, cast_per_tensor_sharded, cast_per_tensor_async

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=180), device_id=dev)

    recipe = bb.Float8CurrentScaling(fp8_format="E4M3")
    batch = args.shard == "batch"
    A, Wt = make_inputs(dev, batch_seed=(1000 + rank) if batch and rank > 0 else None)
    n0, n1 = (0, N) if batch else shard_rows(N, world, rank)
    Wt_sh = Wt[n0:n1].contiguous()
    del Wt
    torch.cuda.synchronize()
    job_flops = FLOPS * (world if batch else 1)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    gemm_events = []

    def step(a_in, w_in, record=False):
        if batch:
            # activations: global amax over all ranks' batches, its all-reduce
            # in flight while the (replicated) weight is cast
            pending = cast_per_tensor_async(a_in, recipe)
            sw = bb.cast(w_in, recipe)
            sa = pending.wait()
        else:
            sa = bb.cast(a_in, recipe)
            sw = cast_per_tensor_sharded(w_in, recipe)
        if record:
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record()
        out = bb.linear(sa, sw, out_dtype=torch.bfloat16)
        if record:
            e1.record()
            gemm_events.append((e0, e1))
        return out

    # ---- device-resident timing
    for _ in range(args.warmup):
        step(A, Wt_sh)
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    uuid = "GPU-" + str(torch.cuda.get_device_properties(dev).uuid) \
        if hasattr(torch.cuda.get_device_properties(dev), "uuid") else None
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    with Clocks(uuid) as clk:
        t_start.record()
        for _ in range(args.steps):
            step(A, Wt_sh, record=True)
        t_end.record()
        torch.cuda.synchronize()
    barrier()
    ms = t_start.elapsed_time(t_end) / args.steps
    gemm_ms = statistics.mean(e0.elapsed_time(e1) for e0, e1 in gemm_events)
    ms_t = torch.tensor([ms, gemm_ms], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
    ms, gemm_ms_max = ms_t.tolist()
    value = job_flops / (ms * 1e-3) / 1e12

    # ---- end to end through the public API, host buffers
    # Every step copies its own inputs from pinned host memory and its result
    # back. The copies run on their own streams and the device buffers are
    # double-buffered, so step i+1's upload and step i-1's download overlap
    # step i's kernels, as in a serving loop.
    e2e = None
    if not args.no_e2e:
        A_h = A.cpu().pin_memory()
        W_h = Wt_sh.cpu().pin_memory()
        out_h = [torch.empty((M, n1 - n0), dtype=torch.bfloat16).pin_memory() for _ in range(2)]
        A_d = [torch.empty_like(A) for _ in range(2)]
        W_d = [torch.empty_like(Wt_sh) for _ in range(2)]
        s_h2d, s_cmp, s_d2h = torch.cuda.Stream(), torch.cuda.Stream(), torch.cuda.Stream()
        ev_in = [torch.cuda.Event() for _ in range(2)]    # inputs of buffer b uploaded
        ev_used = [torch.cuda.Event() for _ in range(2)]  # compute done reading buffer b
        ev_out = [torch.cuda.Event() for _ in range(2)]   # result of buffer b computed
        ev_down = [torch.cuda.Event() for _ in range(2)]  # result of buffer b downloaded
        outs = [None, None]

        def e2e_steps(n):
            for i in range(n):
                b = i & 1
                with torch.cuda.stream(s_h2d):
                    if i >= 2:
                        s_h2d.wait_event(ev_used[b])
                    A_d[b].copy_(A_h, non_blocking=True)
                    W_d[b].copy_(W_h, non_blocking=True)
                    ev_in[b].record(s_h2d)
                with torch.cuda.stream(s_cmp):
                    s_cmp.wait_event(ev_in[b])
                    if i >= 2:
                        s_cmp.wait_event(ev_down[b])  # its output buffer is free
                    outs[b] = step(A_d[b], W_d[b])
                    ev_used[b].record(s_cmp)
                    ev_out[b].record(s_cmp)
                with torch.cuda.stream(s_d2h):
                    s_d2h.wait_event(ev_out[b])
                    out_h[b].copy_(outs[b], non_blocking=True)
                    ev_down[b].record(s_d2h)

        e2e_steps(max(2, args.warmup))
        torch.cuda.synchronize()
        barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(s_h2d)
        s_cmp.wait_stream(s_h2d)
        s_d2h.wait_stream(s_h2d)
        e2e_steps(args.steps)
        s_h2d.wait_stream(s_d2h)
        s_h2d.wait_stream(s_cmp)
        e1.record(s_h2d)
        torch.cuda.synchronize()
        barrier()
        e_ms = torch.tensor([e0.elapsed_time(e1) / args.steps], device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(e_ms, op=dist.ReduceOp.MAX)
        e2e = {"value": job_flops / (e_ms.item() * 1e-3) / 1e12, "unit": "TFLOP/s",
               "h2d_bytes_per_step": A_h.numel() * 2 + W_h.numel() * 2,
               "d2h_bytes_per_step": out_h[0].numel() * 2,
               "ms_per_step": e_ms.item(),
               "pipelining": "uploads, kernels and downloads of consecutive steps overlap "
                             "(3 streams, 2 buffers)"}
        if world > 1:
            hb = torch.tensor([e2e["h2d_bytes_per_step"], e2e["d2h_bytes_per_step"]],
                              device=dev, dtype=torch.float64)
            dist.all_reduce(hb)
            e2e["h2d_bytes_per_step"], e2e["d2h_bytes_per_step"] = [int(v) for v in hb.tolist()]

    # ---- roofline of the dominant kernel (the GEMM), per rank
    peaks, src = measured_peaks()
    peak_fp8 = 2.0 * peaks["bf16_tflops_sustained"]
    gemm_flops_rank = 2.0 * M * (n1 - n0) * K
    achieved = gemm_flops_rank / (gemm_ms * 1e-3) / 1e12
    roofline = {"bound": "tensor", "achieved": achieved, "peak": peak_fp8, "unit": "TFLOP/s",
                "frac": achieved / peak_fp8, "traffic": GEMM_DRAM_BYTES,
                "kernel": "brc::gemm::k_gemm_pair<kPerTensor,E4M3,E4M3,bf16>",
                "peak_source": f"2 x bf16_tflops_sustained of {src} MEASURED_PEAKS.json "
                               "(dense FP8 = 2x dense bf16)",
                "frac_vs_burst": achieved / (2.0 * peaks["bf16_tflops"]),
                "gemm_ms": gemm_ms}

    extras = {}
    if args.per_recipe and world == 1:
        del A, Wt_sh
        torch.cuda.empty_cache()
        extras = per_recipe(peaks, src)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(args)

    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak" if batch else "strong",
            "vs_baseline": None,
            "dtype": "e4m3 x e4m3 -> f32 accumulate -> bf16 out",
            "data": "synthetic (seeded torch generator, BASELINE configs[1] shapes/distributions)",
            "config": {"workload": WORKLOAD, "M": M * (world if batch else 1), "N": N, "K": K,
                       "M_per_gpu": M,
                       "parallelism": "single GPU" if world == 1 else
                       (f"data parallel over {world} GPUs: {M} activation rows per GPU, W "
                        "replicated, one NCCL all-reduce(MAX) of the activations' amax "
                        "(overlapped with the weight cast)") if batch else
                       f"W^T split along N over {world} GPUs, A replicated, "
                       "one NCCL all-reduce(MAX) of the weight amax",
                       "l2": "inputs larger than L2 (A is 268 MB)"},
            "clocks": clk.summary(),
            "e2e": e2e,
            "gpu_launches": 7 * args.steps * world,
            "gpu_launches_per_rank": 7 * args.steps,
            "roofline": roofline,
            "cpu_baseline": cpu,
        }
        if extras:
            line["per_recipe"] = extras
        print(json.dumps(line), flush=True)
    return 0


def _warm_pool(pool, nproc):
    import numpy as np
    list(pool.map(_cpu_encode_rows, [(np.zeros((1, 16), np.float32), 1.0, "E4M3")] * nproc))


def cpu_baseline(args):
    """Rank 0, N = 1: the oracle port of the reference, bounded sample."""
    if args.cpu_rows is None:
        args.cpu_rows = 64
    import multiprocessing as mp
    from concurrent.futures import ProcessPoolExecutor
    A_np, Wt_np = host_inputs_numpy()
    nproc = os.cpu_count() or 1
    with ProcessPoolExecutor(max_workers=nproc, mp_context=mp.get_context("spawn")) as pool:
        _warm_pool(pool, nproc)
        sec, parts = cpu_reference_step(A_np, Wt_np, args.cpu_rows, pool, nproc)
    return {"value": FLOPS / sec / 1e12, "unit": "TFLOP/s", "cores": nproc, "kind": "port",
            "sample": f"{args.cpu_rows} rows of A and of W^T encoded (literal LUT search, "
                      f"{nproc} spawn processes), full-tensor amax, {args.cpu_rows}-row dequant "
                      "+ sgemm; extrapolated linearly by rows",
            "seconds_per_step": sec,
            "breakdown_s": {k: round(v, 3) for k, v in parts.items()}}


# --------------------------------------------------------------- per recipe


def _time_ms(fn, iters=10, warm=3, graph=True):
    """Device time per call. With graph=True the call is captured once in a
    CUDA graph and replayed, so small kernels are timed without the Python
    launch overhead of the wrapper (the GPU would otherwise idle between
    launches); each replay runs the same kernels with the same arguments."""
    import torch
    for _ in range(warm):
        fn()
    torch.cuda.synchronize()
    run = fn
    if graph:
        g = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            with torch.cuda.graph(g, stream=s):
                fn()
        torch.cuda.current_stream().wait_stream(s)
        run = g.replay
        run()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record()
    for _ in range(iters):
        run()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / iters


def per_recipe(peaks, src):
    """Every BASELINE config at full size on one GPU: cast GB/s (algorithmic
    bytes: input read once -- twice for per-tensor, whose global amax must be
    known before any code is written -- plus codes, scales and side outputs
    written) and GEMM TFLOP/s. Inputs exceed L2 except where noted."""
    import torch
    import breccia_b200 as bb
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(1)
    hbm = peaks["hbm_gbs"]
    fp8 = 2.0 * peaks["bf16_tflops_sustained"]
    fp4 = 4.0 * peaks["bf16_tflops_sustained"]
    res = {}

    def cast_entry(name, x, r, bytes_, **kw):
        ms = _time_ms(lambda: bb.cast(x, r, **kw))
        gbs = bytes_ / (ms * 1e-3) / 1e9
        res[name] = {"ms": ms, "GB/s": gbs, "frac_hbm": gbs / hbm}

    def ste_entry(name, x, r, bytes_):
        # fused cast_ste forward vs the unfused cast -> dequantize -> x + (y - x)
        ms = _time_ms(lambda: bb.cast_ste(x, r))
        ms_u = _time_ms(lambda: x + (bb.dequantize(bb.cast(x, r)) - x))
        gbs = bytes_ / (ms * 1e-3) / 1e9
        res[name] = {"ms": ms, "GB/s": gbs, "frac_hbm": gbs / hbm, "unfused_ms": ms_u}

    def gemm_entry(name, a, w, m, n, k, peak):
        ms = _time_ms(lambda: bb.linear(a, w, out_dtype=torch.bfloat16))
        tf = 2.0 * m * n * k / (ms * 1e-3) / 1e12
        res[name] = {"ms": ms, "TFLOP/s": tf, "frac_peak": tf / peak}

    # C1 Float8BlockScaling: A f32 (2048, 7168) 1x128; W^T f32 (4096, 7168) 128x128
    A = torch.randn(2048, 7168, generator=g, device=dev)
    Wt = torch.randn(4096, 7168, generator=g, device=dev) * 0.02
    r = bb.Float8BlockScaling(block_k=128)
    cast_entry("c1_cast_A_block1x128_f32", A, r, A.numel() * 5 + A.numel() // 128 * 4)
    cast_entry("c1_cast_Wt_block128x128_f32", Wt, r, Wt.numel() * 5 + Wt.numel() // 16384 * 4,
               block_m=128)
    ms = _time_ms(lambda: bb.linear(bb.cast(A, r), bb.cast(Wt, r, block_m=128),
                                    out_dtype=torch.float32))
    res["c1_step_cast_both_gemm_block_fp8_f32out"] = {
        "ms": ms, "TFLOP/s": 2.0 * 2048 * 4096 * 7168 / (ms * 1e-3) / 1e12}
    gemm_entry("c1_gemm_block_fp8", bb.cast(A, r), bb.cast(Wt, r, block_m=128), 2048, 4096, 7168,
               fp8)
    del A, Wt
    # C2 per-tensor: A bf16 (16384, 8192): two reads + one write
    A = torch.randn(16384, 8192, generator=g, device=dev).to(torch.bfloat16)
    cast_entry("c2_cast_A_pertensor_bf16", A, bb.Float8CurrentScaling(), A.numel() * 5)
    ste_entry("c2_cast_ste_A_pertensor_bf16", A, bb.Float8CurrentScaling(), A.numel() * 8)
    del A
    # C3 MXFP8: A bf16 (8192, 8192), W^T bf16 (28672, 8192); GEMM 8192 x 28672 x 8192
    r = bb.MXFP8BlockScaling()
    A = torch.randn(8192, 8192, generator=g, device=dev).to(torch.bfloat16)
    Wt = (torch.randn(28672, 8192, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    cast_entry("c3_cast_A_mxfp8_bf16", A, r, A.numel() * 3 + A.numel() // 32 * 2)
    cast_entry("c3_cast_Wt_mxfp8_bf16", Wt, r, Wt.numel() * 3 + Wt.numel() // 32 * 2)
    ste_entry("c3_cast_ste_A_mxfp8_bf16", A, r, A.numel() * 6)
    gemm_entry("c3_gemm_mxfp8", bb.cast(A, r), bb.cast(Wt, r), 8192, 28672, 8192, fp8)
    del A, Wt
    # C4 NVFP4: A bf16 (4096, 8192), W^T bf16 (28672, 8192) Student-t(4) * 0.02
    r = bb.NVFP4BlockScaling()
    A = torch.randn(4096, 8192, generator=g, device=dev).to(torch.bfloat16)
    Wt = (torch.distributions.StudentT(torch.tensor(4.0, device=dev)).sample((28672, 8192))
          * 0.02).to(torch.bfloat16)
    cast_entry("c4_cast_A_nvfp4_bf16", A, r, A.numel() * 3.5 + A.numel() // 16 * 2)
    cast_entry("c4_cast_Wt_nvfp4_bf16", Wt, r, Wt.numel() * 3.5 + Wt.numel() // 16 * 2)
    sw = bb.cast(Wt, r)
    gemm_entry("c4_gemm_nvfp4", bb.cast(A, r), sw, 4096, 28672, 8192, fp4)
    ms = _time_ms(lambda: bb.requantize(sw, bb.MXFP8BlockScaling()))
    n = Wt.numel()
    b = n * 1 + n // 16 + n * 1 + n // 32 * 2
    res["c4_requant_Wt_nvfp4_to_mxfp8"] = {"ms": ms, "GB/s": b / (ms * 1e-3) / 1e9,
                                           "frac_hbm": b / (ms * 1e-3) / 1e9 / hbm}
    # loading the C4 weight from breccia's packed on-disk order (bridges): unpack to
    # codes + tensor-core packed order, and rebuild the scale atoms
    from breccia_b200 import _lib as L
    st_ = torch.cuda.current_stream().cuda_stream
    pk = torch.empty(n // 2, dtype=torch.uint8, device=dev)
    L.call("brc_pack_nibbles_hi", sw.data.data_ptr(), n, pk.data_ptr(), st_)
    codes_ = torch.empty(n, dtype=torch.uint8, device=dev)
    lo_ = torch.empty(n // 2, dtype=torch.uint8, device=dev)
    atoms_ = torch.empty(bb.gemm_operands(sw)["sf_mma"].numel(), dtype=torch.uint8, device=dev)

    def _load_nvfp4():
        s_ = torch.cuda.current_stream().cuda_stream  # the capturing stream under a graph
        L.call("brc_unpack_nibbles_hi", pk.data_ptr(), n, codes_.data_ptr(), lo_.data_ptr(), s_)
        L.call("brc_scale_atoms", sw.scale.data_ptr(), 28672, 8192 // 16, atoms_.data_ptr(), s_)
    ms = _time_ms(_load_nvfp4)
    b = n // 2 + n // 16 + n + n // 2 + atoms_.numel()
    res["c4_load_Wt_nvfp4_from_packed"] = {"ms": ms, "GB/s": b / (ms * 1e-3) / 1e9,
                                           "frac_hbm": b / (ms * 1e-3) / 1e9 / hbm}
    del A, Wt, sw, pk, codes_, lo_, atoms_
    # C5 INT4 asymmetric g128: W^T f32 (28672, 8192)
    Wt = torch.randn(28672, 8192, generator=g, device=dev) * 0.02
    r = bb.INT4Scaling(group_size=128, signed=False, symmetric=False)
    cast_entry("c5_cast_Wt_int4_asym_f32", Wt, r,
               Wt.numel() * 5.5 + Wt.numel() // 128 * 4)
    sw = bb.cast(Wt, r)
    del Wt
    # rebuilding the skinny-GEMM tiles of a stored (loaded) C5 weight
    tl = bb.gemm_operands(sw)
    n = sw.data.numel()

    def _tiles():
        L.call("brc_int4_tiles", sw.data.data_ptr(), 28672, 8192, sw.scale.data_ptr(),
               sw.zero_point.data_ptr(), L.SCALE_F16, tl["int4_tiles"].data_ptr(),
               tl["int4_scale_tiles"].data_ptr(), tl["int4_zp_tiles"].data_ptr(),
               torch.cuda.current_stream().cuda_stream)
    ms = _time_ms(_tiles)
    b = n + n // 128 * 2 * 2 + n // 2 + n // 128 * 4 * 2
    res["c5_int4_tiles_from_stored_Wt"] = {"ms": ms, "GB/s": b / (ms * 1e-3) / 1e9,
                                           "frac_hbm": b / (ms * 1e-3) / 1e9 / hbm}
    for m in (1, 4, 16):
        A = torch.randn(m, 8192, generator=g, device=dev).to(torch.bfloat16)
        ms = _time_ms(lambda: bb.linear(A, sw, out_dtype=torch.bfloat16), iters=50)
        b = 28672 * 8192 // 2 + 2 * (28672 * 64 * 2) + m * 8192 * 2 + m * 28672 * 2
        gbs = b / (ms * 1e-3) / 1e9
        res[f"c5_gemv_int4_M{m}"] = {"ms": ms, "GB/s": gbs, "frac_hbm": gbs / hbm,
                                     "TFLOP/s": 2.0 * m * 28672 * 8192 / (ms * 1e-3) / 1e12}
    del sw
    torch.cuda.empty_cache()
    res["peaks"] = {"hbm_gbs": hbm, "fp8_tflops": fp8, "fp4_tflops": fp4,
                    "source": f"{src} MEASURED_PEAKS.json: hbm_gbs; 2x / 4x "
                              "bf16_tflops_sustained for dense FP8 / FP4"}
    return res


# --------------------------------------------------------------- ncu cases
# Small single-kernel cases for `ncu --set full -k regex:<kernel> -c 3`. Each
# sets up its operands, then launches the kernel 3 times. Operands exceed the
# 126 MB L2 so DRAM counters stay meaningful, and stay far below a GB.

NCU_CASES = {
    "gemm_fp8": "per-tensor FP8 GEMM 8192x8192x8192 (A, B 64 MB each) -> bf16",
    "gemm_mxfp8": "MXFP8 GEMM 8192x8192x8192 -> bf16",
    "gemm_nvfp4": "NVFP4 GEMM 8192x16384x8192 -> bf16",
    "gemm_block": "block-FP8 GEMM 2048x4096x7168 (C1) -> f32",
    "gemv_int4": "INT4 skinny GEMM M=1, W^T 28672x8192 (C5) -> bf16",
    "cast_pertensor": "per-tensor E4M3 cast, bf16 16384x8192 (amax + apply)",
    "cast_mxfp8": "MXFP8 cast, bf16 8192x8192",
    "cast_nvfp4": "NVFP4 cast, bf16 8192x8192",
    "cast_int4": "INT4 asym g128 cast, f32 8192x8192",
    "cast_block2d": "128x128 block FP8 cast, f32 4096x7168",
    "requant_nv_mx": "NVFP4 -> MXFP8 requantize, 8192x8192",
}


def run_ncu_case(name):
    import torch
    import breccia_b200 as bb
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    g = torch.Generator(device=dev).manual_seed(0)

    def bf16(r, c, s=1.0):
        return (torch.randn(r, c, generator=g, device=dev) * s).to(torch.bfloat16)

    if name.startswith("gemm_") and name != "gemm_block":
        r = {"gemm_fp8": bb.Float8CurrentScaling(), "gemm_mxfp8": bb.MXFP8BlockScaling(),
             "gemm_nvfp4": bb.NVFP4BlockScaling()}[name]
        n = 16384 if name == "gemm_nvfp4" else 8192
        a, w = bb.cast(bf16(8192, 8192), r), bb.cast(bf16(n, 8192, 0.02), r)
        fn = lambda: bb.linear(a, w, out_dtype=torch.bfloat16)  # noqa: E731
    elif name == "gemm_block":
        r = bb.Float8BlockScaling()
        a = bb.cast(torch.randn(2048, 7168, generator=g, device=dev), r)
        w = bb.cast(torch.randn(4096, 7168, generator=g, device=dev) * 0.02, r, block_m=128)
        fn = lambda: bb.linear(a, w, out_dtype=torch.float32)  # noqa: E731
    elif name == "gemv_int4":
        r = bb.INT4Scaling(group_size=128, signed=False, symmetric=False)
        w = bb.cast(torch.randn(28672, 8192, generator=g, device=dev) * 0.02, r)
        a = bf16(1, 8192)
        fn = lambda: bb.linear(a, w, out_dtype=torch.bfloat16)  # noqa: E731
    elif name == "requant_nv_mx":
        st = bb.cast(bf16(8192, 8192), bb.NVFP4BlockScaling())
        fn = lambda: bb.requantize(st, bb.MXFP8BlockScaling())  # noqa: E731
    else:
        x, r, kw = {
            "cast_pertensor": (lambda: bf16(16384, 8192), bb.Float8CurrentScaling(), {}),
            "cast_mxfp8": (lambda: bf16(8192, 8192), bb.MXFP8BlockScaling(), {}),
            "cast_nvfp4": (lambda: bf16(8192, 8192), bb.NVFP4BlockScaling(), {}),
            "cast_int4": (lambda: torch.randn(8192, 8192, generator=g, device=dev),
                          bb.INT4Scaling(group_size=128, signed=False, symmetric=False), {}),
            "cast_block2d": (lambda: torch.randn(4096, 7168, generator=g, device=dev),
                             bb.Float8BlockScaling(), {"block_m": 128}),
        }[name]
        xin = x()
        fn = lambda: bb.cast(xin, r, **kw)  # noqa: E731
    torch.cuda.synchronize()
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    print(json.dumps({"ncu_case": name, "what": NCU_CASES[name], "ok": True}))
    return 0


def main():
    args = parse()
    if args.ncu_case:
        return run_ncu_case(args.ncu_case)
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
