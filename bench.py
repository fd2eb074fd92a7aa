#!/usr/bin/env python
"""Benchmark of the INT4 group-quantised decode GEMV on B200.

Workload (one step = one GEMV, i.e. one decode token through one linear):
  x fp32 [1, 4096] ~ N(0,1); W [4096 x 14336] ~ N(0, 0.02) quantised to the
  reference INT4 layout with group 32 along K (asymmetric: fp16 scale + int8
  zero point per group and column, two nibbles per byte); y fp32 [1, 14336].
Weights are packed once on the device by the library's own packer.  Eight
distinct copies of the packed weights (8 x 34.9 MB = 279 MB > 126 MB L2) are
cycled so every step streams its weights from HBM.

Arms:
  (default)          our kernel through the C ABI; value = aggregate HBM GB/s
                     of algorithmic bytes over all ranks (weak scaling: every
                     rank runs the full workload on its own GPU, no collective
                     on the data path).
  --impl reference   the reference's own CPU kernel (matmul_int4_grouped_neon,
                     compiled from its header into oracle/_ref) on all host
                     threads; rank 0 only.

Launch for N > 1: python -m torch.distributed.run --nproc-per-node N bench.py --gpus N
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import ctypes
import json
import math
import os
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "INT4 decode tokens/s & GEMV HBM GB/s; flash-attn TFLOP/s at 1/2/4/8 B200"
K_DIM, N_DIM, GS = 4096, 14336, 32
WORKLOAD = (f"int4_gemv: x fp32 [1,{K_DIM}] x W[{K_DIM}x{N_DIM}] int4 asym group {GS} "
            f"(fp16 scale + int8 zero), y fp32 [1,{N_DIM}]")


def algorithmic_bytes(K=K_DIM, N=N_DIM, gs=GS) -> int:
    G = (K + gs - 1) // gs
    return ((K + 1) // 2) * N + G * N * 2 + G * N * 1 + K * 4 + N * 4


def rank_env():
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("LOCAL_RANK", 0)),
            int(os.environ.get("WORLD_SIZE", 1)))


# ----------------------------------------------------------------------------- process groups
_PG = {"init": False, "gloo": None}


def dist_setup(local_rank):
    """One NCCL group (device-side barriers and max over ranks) and one gloo
    group (host-side exchanges) for the whole run; nothing at world 1."""
    import datetime

    import torch
    import torch.distributed as dist
    _, _, world = rank_env()
    if world == 1 or _PG["init"]:
        return
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=900),
                            device_id=torch.device("cuda", local_rank))
    _PG["gloo"] = dist.new_group(backend="gloo", timeout=datetime.timedelta(seconds=900))
    _PG["init"] = True


def dist_teardown():
    if _PG["init"]:
        import torch.distributed as dist
        dist.destroy_process_group()
        _PG["init"] = False


def dev_barrier(local_rank):
    if _PG["init"]:
        import torch.distributed as dist
        dist.barrier(device_ids=[local_rank])


def dev_max(v, dev):
    """Max over ranks of a device-timed value (NCCL)."""
    if not _PG["init"]:
        return v
    import torch
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def host_barrier():
    if _PG["init"]:
        import torch.distributed as dist
        dist.barrier(group=_PG["gloo"])


def host_max(vals):
    """Element-wise max over ranks of host values (gloo)."""
    if not _PG["init"]:
        return list(vals)
    import torch
    import torch.distributed as dist
    t = torch.tensor(list(vals), dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=_PG["gloo"])
    return [float(x) for x in t]


def host_bcast(obj_list, src=0):
    if _PG["init"]:
        import torch.distributed as dist
        dist.broadcast_object_list(obj_list, src=src, group=_PG["gloo"])


def read_peak_hbm():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as fh:
            return float(json.load(fh)["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def read_profile_traffic():
    """DRAM bytes per launch of the GEMV kernel from the committed ncu summary."""
    path = os.path.join(ROOT, "profiles", "w4_gemv_k4096_n14336_g32.md")
    try:
        for line in open(path):
            if line.startswith("traffic_bytes_per_launch:"):
                return float(line.split(":", 1)[1].strip().split()[0])
    except OSError:
        pass
    return None


class ClockSampler:
    """SM clocks and throttle reasons, sampled during the timed region.

    NVML (pynvml) is polled from a background thread every interval_ms, so
    that a timed region of a few milliseconds still gets samples; without
    pynvml, nvidia-smi -lms does the sampling."""
    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    NAMES = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, gpu_index: int, interval_ms: float = 0.5):
        import threading
        self.proc = None
        self.thread = None
        self.samples = []  # (sm_mhz, sm_max_mhz, reasons)
        self.stop_flag = threading.Event()
        try:
            import pynvml
            import torch
            pynvml.nvmlInit()
            pr = torch.cuda.get_device_properties(gpu_index)
            bus = f"{pr.pci_domain_id:08x}:{pr.pci_bus_id:02x}:{pr.pci_device_id:02x}.0"
            h = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
            masks = {"hw_slowdown": pynvml.nvmlClocksEventReasonHwSlowdown,
                     "hw_thermal_slowdown": pynvml.nvmlClocksEventReasonHwThermalSlowdown,
                     "sw_thermal_slowdown": pynvml.nvmlClocksEventReasonSwThermalSlowdown,
                     "sw_power_cap": pynvml.nvmlClocksEventReasonSwPowerCap}
            smax = float(pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM))

            def poll():
                while not self.stop_flag.is_set():
                    try:
                        sm = float(pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM))
                        r = pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)
                        self.samples.append((sm, smax, {n for n, m in masks.items() if r & m}))
                    except pynvml.NVMLError:
                        return
                    self.stop_flag.wait(interval_ms / 1e3)

            self.thread = threading.Thread(target=poll, daemon=True)
            self.thread.start()
            return
        except Exception:
            self.thread = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(gpu_index), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", str(max(20, int(interval_ms)))],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (OSError, ValueError):
            self.proc = None

    def stop(self):
        if self.thread is not None:
            self.stop_flag.set()
            self.thread.join(timeout=5)
            src = "nvml"
        elif self.proc is not None:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=10)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            for line in out.strip().splitlines():
                parts = [p.strip() for p in line.split(",")]
                if len(parts) < 8:
                    continue
                try:
                    sm, smax = float(parts[0]), float(parts[1])
                except ValueError:
                    continue
                self.samples.append((sm, smax, {n for n, v in zip(self.NAMES, parts[4:8])
                                                if v.lower() in ("active", "1", "yes")}))
            src = "nvidia-smi"
        else:
            return None
        if not self.samples:
            return None
        reasons = set().union(*(r for _, _, r in self.samples))
        return {"sm_mhz": float(np.median([s for s, _, _ in self.samples])),
                "sm_max_mhz": max(m for _, m, _ in self.samples), "reasons": sorted(reasons),
                "samples": len(self.samples), "source": src}


# ----------------------------------------------------------------------------- CPU baseline
def cpu_baseline_sample(seconds=12.0):
    """The reference's own INT4 kernel (oracle/_ref), 1 thread, full config shape."""
    import oracle
    if oracle.ref_available():
        R = oracle.ref()
        fn, kind = R.sgref_neon_matmul_int4_grouped, "reference"
    else:
        fn, kind = None, "port"
    K, N, gs = K_DIM, N_DIM, GS
    rng = np.random.default_rng(7)
    B = rng.integers(0, 256, (K // 2, N), dtype=np.uint8)
    S = (rng.random((K // gs, N)) * 0.01).astype(np.float16)
    Z = rng.integers(-8, 8, (K // gs, N), dtype=np.int8)
    C = np.zeros(N, np.float16)
    P = lambda a: a.ctypes.data_as(ctypes.c_void_p)  # noqa: E731
    if kind == "reference":
        A = rng.integers(-128, 128, K, dtype=np.int8)
        call = lambda: fn(P(A), P(B), P(S), P(Z), P(C), K, N, gs)  # noqa: E731
    else:
        x = rng.standard_normal((1, K)).astype(np.float32)
        call = lambda: oracle.matmul_int4_grouped(x, B, S, Z, K, N, gs)  # noqa: E731
    call()
    n, t0 = 0, time.perf_counter()
    while True:
        call()
        n += 1
        if time.perf_counter() - t0 >= seconds:
            break
    dt = time.perf_counter() - t0
    gbs = n * algorithmic_bytes() / dt / 1e9
    return {"value": round(gbs, 4), "unit": "GB/s", "cores": 1, "kind": kind,
            "sample": f"{n} full GEMV calls (K={K}, N={N}, gs={gs}, int8 activations: the reference "
                      f"INT4 kernel's only activation type) in {dt:.1f} s on 1 host thread"}


# ----------------------------------------------------------------------------- our arm
def shard_columns(N, world, rank):
    """Rank's share of N columns, in whole 128-column strips: (first, count)."""
    strips = N // 128
    per, extra = divmod(strips, world)
    first = (rank * per + min(rank, extra)) * 128
    count = (per + (1 if rank < extra else 0)) * 128
    return first, count


def run_ours(args):
    """The INT4 GEMV (K=4096, N=14336, g32, fp32 x and y).  One GPU: the whole
    GEMV.  N GPUs: its columns split over the ranks (strong scaling, no
    collective on the data path); value = the algorithmic bytes all ranks
    streamed / the slowest rank's time."""
    import torch

    from silicongraph_b200 import _lib, kernels

    rank, local_rank, world = rank_env()
    torch.cuda.set_device(local_rank)
    dist_setup(local_rank)
    lib = _lib.load()
    dev = torch.device("cuda", local_rank)
    K, gs = K_DIM, GS
    G = K // gs
    n0, N = shard_columns(N_DIM, world, rank)
    nbytes = algorithmic_bytes(K, N, gs)
    all_bytes = sum(algorithmic_bytes(K, shard_columns(N_DIM, world, r)[1], gs) for r in range(world))

    # inputs generated on the host, copied; weights packed on the device by our packer
    # (every rank draws the full matrix from one seed and packs its own columns)
    rng = np.random.default_rng(1234)
    W = torch.from_numpy((rng.standard_normal((K, N_DIM)) * 0.02).astype(np.float32)[:, n0:n0 + N].copy()).to(dev)
    x_host = torch.from_numpy(rng.standard_normal((1, K)).astype(np.float32)).pin_memory()
    l2 = torch.cuda.get_device_properties(dev).L2_cache_size
    copies = max(2, math.ceil(2.0 * l2 / (nbytes - K * 4 - N * 4)))
    Bs, Ss, Zs = [], [], []
    stream = torch.cuda.Stream(dev)
    with torch.cuda.stream(stream):
        for _ in range(copies):
            B = torch.empty((K // 2, N), dtype=torch.uint8, device=dev)
            S = torch.empty((G, N), dtype=torch.float16, device=dev)
            Z = torch.empty((G, N), dtype=torch.int8, device=dev)
            _lib.check(lib.sg_quantize_int4_grouped(W.data_ptr(), K, N, gs, 0, B.data_ptr(), S.data_ptr(),
                                                    Z.data_ptr(), stream.cuda_stream))
            Bs.append(B)
            Ss.append(S)
            Zs.append(Z)
    stream.synchronize()
    del W
    x = x_host.to(dev)
    y = torch.empty((1, N), dtype=torch.float32, device=dev)
    # the weights are written once, before the timed launches: they may stream
    # before each launch's dependency wait
    params = [kernels.matmul_params(x, Bs[i], y, M=1, K=K, N=N, scales=Ss[i], zeros=Zs[i], group_size=gs,
                                    flags=_lib.SG_MM_STATIC_WEIGHTS) for i in range(copies)]
    pptr = [ctypes.byref(p) for p in params]
    st = stream.cuda_stream
    fn = lib.sg_matmul_int4_grouped

    def launch(i):
        r = fn(pptr[i % copies], st)
        if r != 0:
            raise _lib.SgError(r, _lib.last_error())

    # warm-up (also allocates the library scratch for this stream, outside capture)
    for i in range(args.warmup):
        launch(i)
    stream.synchronize()

    # every timed launch runs from a CUDA graph: one graph of graph_len launches
    # replayed steps // graph_len times, and one of the remaining steps % graph_len
    graph_len = min(args.graph_len, args.steps)
    if graph_len > copies and graph_len % copies == 1:
        graph_len -= 1  # the last launch of one replay and the first of the next use different copies
    n_rep, n_rem = args.steps // graph_len, args.steps % graph_len
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        for i in range(graph_len):
            launch(i)
    g_rem = None
    if n_rem:
        g_rem = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g_rem, stream=stream):
            for i in range(graph_len, graph_len + n_rem):
                launch(i)
    g.replay()
    if g_rem is not None:
        g_rem.replay()
    stream.synchronize()

    # ---- timed region: exactly K steps
    clocks = ClockSampler(torch.cuda.current_device()) if rank == 0 else None
    dev_barrier(local_rank)
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        # a bounded device delay (about 1 ms) ahead of the start event, so that the
        # host has queued the graph launches before the timed region begins and
        # the GPU does not idle on host launch latency inside it
        torch.cuda._sleep(2_000_000)
        e0.record(stream)
        for _ in range(n_rep):
            g.replay()
        if g_rem is not None:
            g_rem.replay()
        e1.record(stream)
    stream.synchronize()
    torch.cuda.synchronize()
    dev_barrier(local_rank)
    clk = clocks.stop() if clocks else None
    ms_local = e0.elapsed_time(e1)
    ms = dev_max(ms_local, dev)
    value = args.steps * all_bytes / (ms / 1e3) / 1e9
    per_gpu = args.steps * nbytes / (ms_local / 1e3) / 1e9

    # ---- end to end: host x -> device, GEMV through the C ABI, y -> host, every step
    e2e_steps = min(args.steps, args.e2e_steps)
    y_host = torch.empty((1, N), dtype=torch.float32).pin_memory()
    dev_barrier(local_rank)
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        e0.record(stream)
        for i in range(e2e_steps):
            x.copy_(x_host, non_blocking=True)
            launch(i)
            y_host.copy_(y, non_blocking=True)
            stream.synchronize()
        e1.record(stream)
    stream.synchronize()
    dev_barrier(local_rank)
    e2e_ms = dev_max(e0.elapsed_time(e1), dev)
    e2e_value = e2e_steps * all_bytes / (e2e_ms / 1e3) / 1e9

    del g, g_rem
    peak, peak_kind = read_peak_hbm()
    # DRAM traffic per launch cannot be read inside a timed run (it needs an ncu
    # capture); the figure is the committed capture of this kernel at this shape
    # with the default launch heuristics, so it is given for the whole GEMV on
    # one GPU only and dropped when tuning knobs are set
    traffic = None if (args.tuning or world > 1) else read_profile_traffic()
    line = {
        "metric": METRIC,
        "value": round(value, 2),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms / args.steps,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded N(0,1) activations, N(0,0.02) weights, host-generated)",
        "config": {"workload": WORKLOAD, "K": K, "N": N_DIM, "group_size": gs,
                   "bytes_per_step": all_bytes, "weight_copies": copies,
                   "l2": f"{copies} rotating weight copies per GPU ({copies * nbytes / 1e6:.0f} MB > L2 "
                         f"{l2 / 1e6:.0f} MB)",
                   "parallelism": ("one GPU: the whole GEMV" if world == 1 else
                                   f"columns split over {world} GPUs ({N} or fewer of {N_DIM} each, whole "
                                   "128-column strips; no data-path collective)"),
                   "timing": (f"{n_rep} replay(s) of a CUDA graph of {graph_len} launches"
                              + (f" + one graph of {n_rem}" if n_rem else "")
                              + " (every timed launch inside a graph), CUDA events, max over ranks")},
        "roofline": {"bound": "hbm", "achieved": round(per_gpu, 2), "peak": peak, "unit": "GB/s",
                     "frac": round(per_gpu / peak, 4), "peak_source": f"{peak_kind} hbm_gbs",
                     "traffic": traffic,
                     "traffic_source": ("ncu dram__bytes_read.sum + dram__bytes_write.sum of one launch at this "
                                        "shape, default heuristics (profiles/w4_gemv_k4096_n14336_g32.md); not "
                                        "measured in this run") if traffic else None,
                     "achieved_basis": ("algorithmic bytes per launch x launches / event time of back-to-back "
                                        "launches (includes inter-launch gaps)"
                                        + ("" if world == 1 else "; rank 0's shard and time"))},
        "e2e": {"value": round(e2e_value, 3), "unit": "GB/s", "steps": e2e_steps,
                "h2d_bytes_per_step": int(x_host.numel() * 4) * world,
                "d2h_bytes_per_step": int(N_DIM * 4)},
        "gpu_launches": args.steps,
        "clocks": clk,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            line["cpu_baseline"] = cpu_baseline_sample(args.cpu_seconds)
        except Exception as e:  # the baseline is reported, never required
            line["cpu_baseline"] = {"value": None, "error": str(e)[:200]}
    return line


# ----------------------------------------------------------------------------- prefill GEMM workloads
PF_M, PF_K, PF_N, PF_GS = 2048, 2048, 8192, 64
PF_WORKLOADS = {
    "prefill_int4": (f"prefill dequant-GEMM: A bf16 [{PF_M},{PF_K}] x W[{PF_K}x{PF_N}] int4 symmetric group {PF_GS} "
                     f"(fp16 scales), C bf16 [{PF_M},{PF_N}]"),
    "prefill_int8": (f"prefill dequant-GEMM: A bf16 [{PF_M},{PF_K}] x W[{PF_K}x{PF_N}] int8 per-channel "
                     f"(f32 scales), C bf16 [{PF_M},{PF_N}]"),
}


def read_peak_tensor():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as fh:
            return float(json.load(fh)["bf16_tflops"]), "measured bf16_tflops (burst)"
    except Exception:
        return 1590.0, "fallback"


def prefill_cpu_sample(kind, seconds):
    """CPU baseline for the prefill GEMM: the reference's own INT4 kernel
    (one activation row per call, int8 activations) looped over sampled rows,
    or the oracle's INT8 per-channel restatement; 1 thread."""
    import oracle
    M, K, N, gs = PF_M, PF_K, PF_N, PF_GS
    rng = np.random.default_rng(5)
    P = lambda a: a.ctypes.data_as(ctypes.c_void_p)  # noqa: E731
    if kind == "prefill_int4":
        B = rng.integers(0, 256, (K // 2, N), dtype=np.uint8)
        S = (rng.random((K // gs, N)) * 0.01).astype(np.float16)
        A = rng.integers(-128, 128, (M, K), dtype=np.int8)
        C = np.zeros(N, np.float16)
        if oracle.ref_available():
            fn, src = oracle.ref().sgref_neon_matmul_int4_grouped, "reference"
            call = lambda m: fn(P(A[m]), P(B), P(S), None, P(C), K, N, gs)  # noqa: E731
        else:
            src = "port"
            call = lambda m: oracle.matmul_int4_grouped(A[m:m + 1], B, S, None, K, N, gs)  # noqa: E731
        what = "reference INT4 kernel (int8 activations, its only activation type), one row per call"
    else:
        B = rng.integers(-128, 128, (K, N), dtype=np.int8)
        s = (rng.random(N) * 1e-3).astype(np.float32)
        A = oracle.f32_to_bf16_bits(rng.standard_normal((M, K)).astype(np.float32))
        src = "port"
        call = lambda m: oracle.gemm_w8_channel(A[m:m + 1], B, s, 1, K, N, a_bf16=True)  # noqa: E731
        what = "oracle INT8 per-channel GEMM (restated GLSL gemm_int8 for bf16 activations), one row per call"
    call(0)
    n, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < seconds:
        call(n % M)
        n += 1
    dt = time.perf_counter() - t0
    tflops = n * 2.0 * K * N / dt / 1e12
    return {"value": round(tflops, 6), "unit": "TFLOP/s", "cores": 1, "kind": src,
            "sample": f"{n} rows of the [{M},{K}]x[{K},{N}] GEMM ({what}) in {dt:.1f} s on 1 host thread"}


def run_prefill(args):
    import torch
    import torch.distributed as dist

    from silicongraph_b200 import _lib, kernels

    rank, local_rank, world = rank_env()
    torch.cuda.set_device(local_rank)
    dist_setup(local_rank)
    lib = _lib.load()
    dev = torch.device("cuda", local_rank)
    M, K, N, gs = PF_M, PF_K, PF_N, PF_GS
    int4 = args.workload == "prefill_int4"
    flops = 2.0 * M * K * N
    rng = np.random.default_rng(4321 + rank)
    a_host = torch.from_numpy(rng.standard_normal((M, K)).astype(np.float32)).to(torch.bfloat16).pin_memory()
    W = torch.from_numpy((rng.standard_normal((K, N)) * 0.02).astype(np.float32)).to(dev)
    stream = torch.cuda.Stream(dev)
    st = stream.cuda_stream
    A = a_host.to(dev)
    A16 = A.half()  # the same activations in the operand type: the GEMM kernel alone
    C = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
    if int4:
        B = torch.empty((K // 2, N), dtype=torch.uint8, device=dev)
        S = torch.empty((K // gs, N), dtype=torch.float16, device=dev)
        _lib.check(lib.sg_quantize_int4_grouped(W.data_ptr(), K, N, gs, 1, B.data_ptr(), S.data_ptr(), None, st))
        stream.synchronize()
        p_main = kernels.matmul_params(A, B, C, M=M, K=K, N=N, scales=S, group_size=gs)
        p_kern = kernels.matmul_params(A16, B, C, M=M, K=K, N=N, scales=S, group_size=gs)
        fn = lib.sg_matmul_int4_grouped
        launches = 2  # activation conversion + GEMM
        dtype = "f16"
    else:
        sc = (W.abs().amax(dim=0) / 127.0).clamp_min(1e-12)
        B = torch.clamp(torch.round(W / sc), -127, 127).to(torch.int8)
        S = sc.float().contiguous()
        p_main = kernels.matmul_params(A, B, C, M=M, K=K, N=N, scales=S)
        p_kern = p_main
        fn = lib.sg_matmul_int8_channel
        launches = 1
        dtype = "bf16"
    del W
    l2 = torch.cuda.get_device_properties(dev).L2_cache_size
    flush = torch.empty(max(2 * l2, 256 << 20), dtype=torch.uint8, device=dev)

    def call(p):
        r = fn(ctypes.byref(p), st)
        if r != 0:
            raise _lib.SgError(r, _lib.last_error())

    def timed(p, steps):
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
        with torch.cuda.stream(stream):
            for e0, e1 in ev:
                flush.zero_()  # L2 flushed between timed steps
                e0.record(stream)
                call(p)
                e1.record(stream)
        stream.synchronize()
        return sum(e0.elapsed_time(e1) for e0, e1 in ev)

    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            call(p_main)
            call(p_kern)
    stream.synchronize()

    def barrier():
        dev_barrier(local_rank)

    def max_over_ranks(v):
        return dev_max(v, dev)

    clocks = ClockSampler(torch.cuda.current_device()) if rank == 0 else None
    barrier()
    torch.cuda.synchronize()
    ms = max_over_ranks(timed(p_main, args.steps))
    ms_kern = max_over_ranks(timed(p_kern, args.steps)) if int4 else ms
    torch.cuda.synchronize()
    barrier()
    clk = clocks.stop() if clocks else None
    value = world * args.steps * flops / (ms / 1e3) / 1e12
    kern_tflops = args.steps * flops / (ms_kern / 1e3) / 1e12

    # end to end: host activations -> device, GEMM through the C ABI, C -> host, every step
    e2e_steps = max(1, min(args.steps, 10))
    c_host = torch.empty((M, N), dtype=torch.bfloat16).pin_memory()
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(e2e_steps):
            A.copy_(a_host, non_blocking=True)
            call(p_main)
            c_host.copy_(C, non_blocking=True)
        e1.record(stream)
    stream.synchronize()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1))
    e2e_value = world * e2e_steps * flops / (e2e_ms / 1e3) / 1e12
    peak, peak_src = read_peak_tensor()
    line = {
        "metric": "prefill dequant-GEMM TFLOP/s (" + ("INT4 g64 symmetric" if int4 else "INT8 per-channel") + ")",
        "value": round(value, 2), "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": dtype,
        "data": "synthetic (seeded N(0,1) activations, N(0,0.02) weights, host-generated)",
        "config": {"workload": PF_WORKLOADS[args.workload], "M": M, "K": K, "N": N,
                   "group_size": gs if int4 else None, "flops_per_step": flops,
                   "l2": "flushed (256 MB write) before every timed step",
                   "parallelism": f"replicas x{world} (no data-path collective)",
                   "timing": "CUDA events around each step, summed; max over ranks"},
        "roofline": {"bound": "tensor", "achieved": round(kern_tflops, 2), "peak": peak, "unit": "TFLOP/s",
                     "frac": round(kern_tflops / peak, 4), "peak_source": peak_src, "traffic": None,
                     "achieved_basis": "algorithmic FLOPs / event time of the GEMM kernel alone "
                     + ("(fp16 activations, no conversion launch)" if int4 else "")},
        "e2e": {"value": round(e2e_value, 3), "unit": "TFLOP/s", "steps": e2e_steps,
                "h2d_bytes_per_step": int(a_host.numel() * 2), "d2h_bytes_per_step": int(c_host.numel() * 2)},
        "gpu_launches": args.steps * launches,
        "clocks": clk,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            line["cpu_baseline"] = prefill_cpu_sample(args.workload, args.cpu_seconds)
        except Exception as e:  # the baseline is reported, never required
            line["cpu_baseline"] = {"value": None, "error": str(e)[:200]}
    return line


# ----------------------------------------------------------------------------- attention workloads
ATTN_WORKLOADS = {
    # name: (B, H, Hkv, S, D, dtype, description)
    "attn_prefill": (1, 28, 4, 8192, 128, "bf16",
                     "causal flash attention, Qwen2.5-7B prefill layer: Q bf16 [1,28,8192,128], "
                     "K/V bf16 [1,4,8192,128] (GQA 7), scale 1/sqrt(128)"),
    "attn_small": (1, 32, 32, 512, 64, "f32",
                   "causal flash attention: Q/K/V fp32 [1,32,512,64], scale 1/8 (CPU-runnable case)"),
}


def attn_flops(H, S, D):
    """Causal: each query attends to itself and the keys before it; QK^T and PV
    cost 2 * D each per (query, key) pair."""
    return 4.0 * H * D * S * (S + 1) / 2


def attn_cpu_sample(seconds):
    """The reference's own flash_attention_fp16 (oracle/_ref) on one head of the
    long-sequence shape at 2048 tokens (1 thread); the oracle port if it is absent."""
    import oracle
    S, D = 2048, 128
    rng = np.random.default_rng(9)
    q, k, v = (rng.standard_normal((1, 1, S, D)).astype(np.float16) for _ in range(3))
    o = np.zeros_like(q)
    P = lambda a: a.ctypes.data_as(ctypes.c_void_p)  # noqa: E731
    if oracle.ref_available():
        fn, kind = oracle.ref().sgref_neon_flash_attention_fp16, "reference"
        call = lambda: fn(P(q), P(k), P(v), P(o), 1, S, 1, 1, D, 0.0, 1)  # noqa: E731
    else:
        kind = "port"
        call = lambda: oracle.flash_attention(q, k, v, causal=True)  # noqa: E731
    n, t0 = 0, time.perf_counter()
    while True:
        call()
        n += 1
        if time.perf_counter() - t0 >= seconds:
            break
    dt = time.perf_counter() - t0
    return {"value": round(n * attn_flops(1, S, D) / dt / 1e12, 6), "unit": "TFLOP/s", "cores": 1, "kind": kind,
            "sample": f"{n} calls of flash_attention_fp16 on one head, S={S}, D={D}, causal, fp16, in {dt:.1f} s "
                      f"on 1 host thread"}


def run_attention(args):
    import torch
    import torch.distributed as dist

    from silicongraph_b200 import _lib, kernels

    rank, local_rank, world = rank_env()
    torch.cuda.set_device(local_rank)
    dist_setup(local_rank)
    lib = _lib.load()
    dev = torch.device("cuda", local_rank)
    B, H, Hkv, S, D, dts, desc = ATTN_WORKLOADS[args.workload]
    tdt = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}[dts]
    flops = attn_flops(H, S, D) * B
    rng = np.random.default_rng(77 + rank)
    hq = torch.from_numpy(rng.standard_normal((B, H, S, D)).astype(np.float32)).to(tdt).pin_memory()
    hk = torch.from_numpy(rng.standard_normal((B, Hkv, S, D)).astype(np.float32)).to(tdt).pin_memory()
    hv = torch.from_numpy(rng.standard_normal((B, Hkv, S, D)).astype(np.float32)).to(tdt).pin_memory()
    Q, K, V = hq.to(dev), hk.to(dev), hv.to(dev)
    O = torch.empty_like(Q)
    stream = torch.cuda.Stream(dev)
    st = stream.cuda_stream
    from silicongraph_b200._lib import SgFlashAttentionParams
    p = SgFlashAttentionParams()
    p.Q, p.K, p.V, p.O = Q.data_ptr(), K.data_ptr(), V.data_ptr(), O.data_ptr()
    p.B, p.S, p.num_heads, p.num_kv_heads, p.head_dim = B, S, H, Hkv, D
    p.causal = 1
    p.io_dtype = kernels.dtype_code(tdt)
    p.S_kv = S
    p.q_pos0 = 0
    l2 = torch.cuda.get_device_properties(dev).L2_cache_size
    flush = torch.empty(max(2 * l2, 256 << 20), dtype=torch.uint8, device=dev)

    def call():
        r = lib.sg_flash_attention(ctypes.byref(p), st)
        if r != 0:
            raise _lib.SgError(r, _lib.last_error())

    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            call()
    stream.synchronize()

    def max_over_ranks(v):
        return dev_max(v, dev)

    clocks = ClockSampler(torch.cuda.current_device()) if rank == 0 else None
    dev_barrier(local_rank)
    torch.cuda.synchronize()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    with torch.cuda.stream(stream):
        for e0, e1 in ev:
            flush.zero_()  # L2 flushed between timed steps
            e0.record(stream)
            call()
            e1.record(stream)
    stream.synchronize()
    ms = max_over_ranks(sum(e0.elapsed_time(e1) for e0, e1 in ev))
    clk = clocks.stop() if clocks else None
    value = world * args.steps * flops / (ms / 1e3) / 1e12
    per_gpu = args.steps * flops / (ms / 1e3) / 1e12
    # end to end: host Q/K/V -> device, attention through the C ABI, O -> host, every step
    e2e_steps = max(1, min(args.steps, 5))
    ho = torch.empty_like(hq).pin_memory()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(e2e_steps):
            Q.copy_(hq, non_blocking=True)
            K.copy_(hk, non_blocking=True)
            V.copy_(hv, non_blocking=True)
            call()
            ho.copy_(O, non_blocking=True)
        e1.record(stream)
    stream.synchronize()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1))
    peak, peak_src = read_peak_tensor()
    esz = Q.element_size()
    line = {
        "metric": "flash-attn TFLOP/s (causal, " + dts + ")",
        "value": round(value, 2), "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": dts, "data": "synthetic (seeded N(0,1) Q/K/V, host-generated)",
        "config": {"workload": desc, "B": B, "H": H, "Hkv": Hkv, "S": S, "D": D,
                   "flops_per_step": flops, "flop_count": "4*H*D*S*(S+1)/2 (causal)",
                   "l2": "flushed (256 MB write) before every timed step",
                   "parallelism": f"replicas x{world} (no data-path collective)",
                   "timing": "CUDA events around each step, summed; max over ranks"},
        "roofline": {"bound": "tensor", "achieved": round(per_gpu, 2), "peak": peak, "unit": "TFLOP/s",
                     "frac": round(per_gpu / peak, 4), "peak_source": peak_src, "traffic": None,
                     "achieved_basis": "algorithmic FLOPs / event time of one sg_flash_attention call"},
        "e2e": {"value": round(world * e2e_steps * flops / (e2e_ms / 1e3) / 1e12, 3), "unit": "TFLOP/s",
                "steps": e2e_steps, "h2d_bytes_per_step": int((hq.numel() + hk.numel() + hv.numel()) * esz),
                "d2h_bytes_per_step": int(ho.numel() * esz)},
        # bf16: V to fp16 + attention; f32: absolute maxima + scaled fp16 copies + attention
        "gpu_launches": args.steps * {"bf16": 2, "f32": 3}.get(dts, 1),
        "clocks": clk,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            line["cpu_baseline"] = attn_cpu_sample(args.cpu_seconds)
        except Exception as e:  # the baseline is reported, never required
            line["cpu_baseline"] = {"value": None, "error": str(e)[:200]}
    return line


# ----------------------------------------------------------------------------- end-to-end decode
DECODE_CFG = dict(layers=16, hidden=2048, heads=32, kv_heads=8, head_dim=64, ffn=8192, vocab=128256,
                  rope_theta=500000.0)
DECODE_WORKLOAD = ("Llama-3.2-1B-shape decoder through the armcc SDK: 16 layers, hidden 2048, 32/8 heads, "
                   "head_dim 64, SwiGLU 8192, vocab 128256, INT4 group-32 weights (lm_head included), fp16 "
                   "activations and KV cache; a prompt of 512 random ids per sequence, then greedy decode")


def build_decode_package(path, cfg, seed=0, gs=32, max_context=1024, max_prefill_chunk=512,
                         model_id="synthetic/llama-3.2-1b-shape"):
    """Random N(0, 0.02) weights (norms 1 + N(0, 0.02)) drawn on the GPU and
    packed by the library's device packer, written as a directory package."""
    from silicongraph_b200 import armpack
    t = armpack.random_cuda_tensors_on_device(cfg, seed=seed, group_size=gs)
    armpack.write_package(path, cfg, t, group_size=gs, max_context=max_context, max_prefill_chunk=max_prefill_chunk,
                          as_zip=False, model_id=model_id)
    H = cfg["hidden_size"]
    weight_bytes = sum(a.nbytes for k, a in t.items() if k != "embed_tokens") + H * 2
    return weight_bytes, t


def decode_cpu_sample(cfg, tensors, seconds):
    """The decoder composition oracle (reference kernel semantics, 1 thread) on
    the same packed model: a 4-token prompt and greedy steps until `seconds`."""
    from oracle.decoder import DecoderOracle
    ref = DecoderOracle(cfg, tensors, group_size=32)
    ref.forward([1, 2, 3, 4])
    n, tok, t0 = 0, 5, time.perf_counter()
    while time.perf_counter() - t0 < seconds:
        tok = int(np.argmax(ref.forward([tok])))
        n += 1
    dt = time.perf_counter() - t0
    return {"value": round(n / dt, 4), "unit": "tokens/s", "cores": 1, "kind": "port",
            "sample": f"{n} greedy decode steps of the full model after a 4-token prompt, decoder composition "
                      f"of the oracle kernels (fp16 values between ops), {dt:.1f} s on 1 host thread"}


def run_decode(args):
    import tempfile

    import torch

    from silicongraph_b200 import armpack, sdk

    import datetime

    import torch.distributed as dist

    rank, local_rank, world = rank_env()
    tp = args.workload == "decode_llama1b_tp"
    torch.cuda.set_device(local_rank)
    os.environ["SG_DEVICE"] = str(local_rank)
    dist_setup(local_rank)  # host-side exchanges (the NCCL id of a tensor-parallel session, max over ranks) on gloo
    c = DECODE_CFG
    cfg = armpack.llama_config(layers=c["layers"], hidden=c["hidden"], heads=c["heads"], kv_heads=c["kv_heads"],
                               head_dim=c["head_dim"], ffn=c["ffn"], vocab=c["vocab"], rope_theta=c["rope_theta"])
    prompt_len = 512
    steps = args.steps
    seed_rank = 0 if tp else rank  # the ranks of one tensor-parallel model share its weights and prompt
    tp_arg = None
    if tp:
        uid = [sdk.tp_unique_id() if rank == 0 else None]
        host_bcast(uid)
        tp_arg = (rank, world, uid[0])
    with tempfile.TemporaryDirectory() as td:
        pkg_path = os.path.join(td, "llama1b_int4")
        weight_bytes, tensors = build_decode_package(pkg_path, cfg, seed=11 + seed_rank,
                                                     max_context=prompt_len + steps + args.warmup + 32)
        rng = np.random.default_rng(5 + seed_rank)
        B = args.batch
        prompt = rng.integers(0, c["vocab"], (B, prompt_len)).astype(np.int32)
        with sdk.Package(pkg_path) as pkg:
            graph = pkg.select(context_length=prompt_len + steps + args.warmup + 24)
            with graph.session(tp=tp_arg, batch=B) as s:
                if B == 1:
                    prefill, decode = (lambda: s.prefill(prompt[0])), (lambda: s.decode().next_token_id)
                else:
                    prefill, decode = (lambda: s.batch_prefill(prompt)), (lambda: int(s.batch_decode()[0]))
                # warm-up: a full prompt and a few steps (allocations, tensor maps, caches)
                prefill()
                for _ in range(args.warmup):
                    decode()
                s.reset()
                clocks = ClockSampler(torch.cuda.current_device(), interval_ms=5) if rank == 0 else None
                host_barrier()
                t0 = time.perf_counter()
                prefill()
                first = decode()                        # the token predicted by the prompt
                t1 = time.perf_counter()
                for _ in range(steps):
                    decode()
                t2 = time.perf_counter()
                clk = clocks.stop() if clocks else None
                # the device time of a step (CUDA events around it), after the timed region
                s.step_gpu_ms(True)
                for _ in range(16):
                    decode()
                gpu_ms = s.step_gpu_ms(False)
                graph_kernels = s.graph_kernels
    decode_s, ttft_s = host_max([t2 - t1, t1 - t0])  # the slowest rank
    tps = steps / decode_s
    seqs = args.batch * (1 if tp else world)  # sequences decoded at once over the whole job
    ctx_mid = prompt_len + steps / 2
    kv_read = 2 * c["layers"] * c["kv_heads"] * c["head_dim"] * 2 * ctx_mid
    bytes_per_token = weight_bytes + kv_read
    bytes_per_step = weight_bytes + args.batch * kv_read  # one step reads the weights once for the whole batch
    peak, peak_src = read_peak_hbm()
    line = {
        "metric": f"INT4 decode tokens/s (Llama-3.2-1B shape, batch {args.batch})",
        "value": round(seqs * tps, 2), "unit": "tokens/s", "n_gpus": world, "steps": steps,
        "warmup": args.warmup, "ms_per_step": 1e3 * decode_s / steps, "higher_is_better": True,
        "scaling": "strong" if tp else "weak", "vs_baseline": None, "dtype": "f16",
        "data": "synthetic (random N(0,0.02) weights drawn on the GPU, random prompt ids)",
        "config": {"workload": DECODE_WORKLOAD, "batch": args.batch, "prompt": prompt_len, "decode_steps": steps,
                   "ttft_ms": round(1e3 * ttft_s, 3), "prefill_tokens_per_s": round(prompt_len / ttft_s, 1),
                   "bytes_per_token": int(bytes_per_token),
                   "gpu_ms_per_step": round(gpu_ms, 4),
                   "parallelism": (f"tensor-parallel x{world} (one session over {world} GPUs, NCCL all-reduce "
                                   "after the o and down projections)") if tp else
                                  f"replicas x{world} (one session per GPU)",
                   "timing": "host clock around armsess_decode calls (each returns the token to the host), "
                             "max over ranks"},
        "roofline": {"bound": "hbm", "achieved": round(bytes_per_step * tps / 1e9 / (world if tp else 1), 2),
                     "peak": peak, "unit": "GB/s",
                     "frac": round(bytes_per_step * tps / 1e9 / (world if tp else 1) / peak, 4),
                     "peak_source": f"{peak_src} hbm_gbs", "traffic": None,
                     "achieved_basis": "(weights + KV cache of every sequence) bytes per step x steps/s, per GPU"},
        "e2e": {"value": round(seqs * tps, 2), "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 8},
        # this library's kernel nodes in the captured decode step (counted in the graph; NCCL's excluded)
        "gpu_launches": steps * graph_kernels if graph_kernels > 0 else None,
        "clocks": clk,
        "first_token": int(first),
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            line["cpu_baseline"] = decode_cpu_sample(cfg, tensors, args.cpu_seconds)
        except Exception as e:  # the baseline is reported, never required
            line["cpu_baseline"] = {"value": None, "error": str(e)[:200]}
    return line


# ----------------------------------------------------------------------------- Qwen-7B shape, tensor-parallel
QWEN_CFG = dict(layers=28, hidden=3584, heads=28, kv_heads=4, head_dim=128, ffn=18944, vocab=152064,
                rope_theta=1000000.0)
QWEN_GS = 128
QWEN_PROMPT = 8192
QWEN_WORKLOAD = ("Qwen2.5-7B-shape decoder through the armcc SDK, tensor-parallel over all ranks: 28 layers, "
                 "hidden 3584, 28/4 heads, head_dim 128, SwiGLU 18944, vocab 152064, INT4 group-128 weights "
                 "(lm_head included); an 8192-token prefill of random ids per sequence, then greedy decode "
                 "of every sequence in lockstep (--batch sequences, 32 in the configuration)")


def run_qwen(args):
    import datetime
    import shutil

    import torch
    import torch.distributed as dist

    from silicongraph_b200 import armpack, sdk

    rank, local_rank, world = rank_env()
    torch.cuda.set_device(local_rank)
    os.environ["SG_DEVICE"] = str(local_rank)
    dist_setup(local_rank)
    c = QWEN_CFG
    cfg = armpack.llama_config(layers=c["layers"], hidden=c["hidden"], heads=c["heads"], kv_heads=c["kv_heads"],
                               head_dim=c["head_dim"], ffn=c["ffn"], vocab=c["vocab"], rope_theta=c["rope_theta"])
    steps = args.steps
    B = args.batch
    ctx = QWEN_PROMPT + steps + args.warmup + 24  # + 16 steps timed on the device after the timed region
    # prompt chunk per forward pass: the whole prompt for one sequence; about 32 K tokens per
    # pass when batched (the activation buffers scale with sequences x chunk)
    chunk = QWEN_PROMPT if B == 1 else max(256, (32768 // B) // 256 * 256)
    # one package on the host's disk, written by rank 0, read by every rank
    root = os.environ.get("SG_BENCH_TMP", "/tmp")
    pkg_path = [os.path.join(root, f"sg_qwen7b_{os.getpid()}") if rank == 0 else None]
    uid = [sdk.tp_unique_id() if rank == 0 else None]
    host_bcast(pkg_path)
    host_bcast(uid)
    pkg_path = pkg_path[0]
    try:
        if rank == 0:
            weight_bytes, _ = build_decode_package(pkg_path, cfg, seed=21, gs=QWEN_GS, max_context=ctx,
                                                   max_prefill_chunk=chunk,
                                                   model_id="synthetic/qwen2.5-7b-shape")
            torch.cuda.empty_cache()
        else:
            weight_bytes = 0
        wb = [weight_bytes]
        host_bcast(wb)
        weight_bytes = wb[0]
        prompt = np.random.default_rng(6).integers(0, c["vocab"], (B, QWEN_PROMPT)).astype(np.int32)
        with sdk.Package(pkg_path) as pkg:
            graph = pkg.select(context_length=ctx)
            with graph.session(tp=(rank, world, uid[0]), batch=B) as s:
                if B == 1:
                    prefill, decode = (lambda p: s.prefill(p[0])), (lambda: s.decode().next_token_id)
                else:
                    prefill, decode = s.batch_prefill, (lambda: int(s.batch_decode()[0]))
                prefill(prompt[:, :1024])          # warm-up: allocations, tensor maps, graph capture
                for _ in range(args.warmup):
                    decode()
                s.reset()
                clocks = ClockSampler(torch.cuda.current_device(), interval_ms=5) if rank == 0 else None
                host_barrier()
                t0 = time.perf_counter()
                prefill(prompt)
                first = decode()
                t1 = time.perf_counter()
                for _ in range(steps):
                    decode()
                t2 = time.perf_counter()
                clk = clocks.stop() if clocks else None
                # the device time of a step (CUDA events around it), after the timed region
                s.step_gpu_ms(True)
                for _ in range(16):
                    decode()
                gpu_ms = s.step_gpu_ms(False)
    finally:
        host_barrier()
        if rank == 0:
            shutil.rmtree(pkg_path, ignore_errors=True)
    ttft_s, decode_s = host_max([t1 - t0, t2 - t1])
    H, L, F, V, D = c["hidden"], c["layers"], c["ffn"], c["vocab"], c["head_dim"]
    Hq, Hkv = c["heads"], c["kv_heads"]
    lin_params = L * (H * (Hq + 2 * Hkv) * D + Hq * D * H + H * 2 * F + F * H)
    S = QWEN_PROMPT
    # linears, causal attention, LM head (last token), per sequence
    flops = B * (2.0 * lin_params * S + L * 4.0 * Hq * D * S * (S + 1) / 2 + 2.0 * H * V)
    prefill_tps = B * S / ttft_s
    achieved = flops / ttft_s / 1e12 / world
    peak, peak_src = read_peak_tensor()
    dec_tps = B * steps / decode_s
    line = {
        "metric": f"Qwen-7B-shape INT4 prefill tokens/s (8192-token prompt{'s x ' + str(B) if B > 1 else ''}, "
                  "tensor-parallel)",
        "value": round(prefill_tps, 1), "unit": "tokens/s", "n_gpus": world, "steps": steps,
        "warmup": args.warmup, "ms_per_step": 1e3 * decode_s / steps, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f16",
        "data": "synthetic (random N(0,0.02) weights drawn on the GPU, random prompt ids)",
        "config": {"workload": QWEN_WORKLOAD, "batch": B, "prompt": S, "prefill_chunk": chunk,
                   "ttft_ms": round(1e3 * ttft_s, 2),
                   "decode_steps": steps, "decode_tokens_per_s": round(dec_tps, 2),
                   "decode_ms_per_token": round(1e3 * decode_s / steps, 3),
                   "decode_gpu_ms_per_step": round(gpu_ms, 4),
                   "weight_bytes": int(weight_bytes), "flops_prefill": flops,
                   "parallelism": f"tensor-parallel x{world} (NCCL all-reduce after o and down)",
                   "timing": "host clock around armsess_prefill / armsess_decode, max over ranks"},
        "roofline": {"bound": "tensor", "achieved": round(achieved, 1), "peak": peak, "unit": "TFLOP/s",
                     "frac": round(achieved / peak, 4), "peak_source": peak_src, "traffic": None,
                     "achieved_basis": "prefill FLOPs (linears + causal attention + LM head) / TTFT, per GPU"},
        "e2e": {"value": round(prefill_tps, 1), "unit": "tokens/s", "h2d_bytes_per_step": B * S * 4,
                "d2h_bytes_per_step": 8 if B == 1 else 4 * B},
        "gpu_launches": None,
        "clocks": clk,
        "first_token": int(first),
    }
    return line


# ----------------------------------------------------------------------------- reference arm
def run_reference(args):
    rank, _, world = rank_env()
    if rank != 0:
        return
    import oracle
    K, N, gs = K_DIM, N_DIM, GS
    if oracle.ref_available():
        fn, kind = oracle.ref().sgref_neon_matmul_int4_grouped, "reference"
    else:
        fn, kind = None, "port"
    threads = os.cpu_count() or 1
    rng = np.random.default_rng(7)
    B = rng.integers(0, 256, (K // 2, N), dtype=np.uint8)
    S = (rng.random((K // gs, N)) * 0.01).astype(np.float16)
    Z = rng.integers(-8, 8, (K // gs, N), dtype=np.int8)
    A = rng.integers(-128, 128, K, dtype=np.int8)
    xf = rng.standard_normal((1, K)).astype(np.float32)
    Cs = [np.zeros(N, np.float16) for _ in range(threads)]
    base = [a.ctypes.data for a in (A, B, S, Z)]

    def slice_call(t, k0, rows):
        if kind == "reference":
            fn(ctypes.c_void_p(base[0] + k0), ctypes.c_void_p(base[1] + (k0 // 2) * N),
               ctypes.c_void_p(base[2] + (k0 // gs) * N * 2), ctypes.c_void_p(base[3] + (k0 // gs) * N),
               Cs[t].ctypes.data_as(ctypes.c_void_p), rows, N, gs)
        else:
            sl = slice(k0 // gs, (k0 + rows) // gs)
            oracle.matmul_int4_grouped(xf[:, k0:k0 + rows], B[k0 // 2:(k0 + rows) // 2], S[sl], Z[sl], rows, N, gs)

    pool = cf.ThreadPoolExecutor(threads)
    units = K // gs  # slices are whole groups

    def step(rows_per_thread, s):
        futs = []
        for t in range(threads):
            k0 = ((s * threads + t) * rows_per_thread) % K
            k0 = min(k0, K - rows_per_thread)
            futs.append(pool.submit(slice_call, t, k0, rows_per_thread))
        for f in futs:
            f.result()

    # calibrate: per-thread slice size so the whole run stays within the time budget
    rows = gs
    t0 = time.perf_counter()
    step(rows, 0)
    t_unit = max(time.perf_counter() - t0, 1e-5)
    budget = args.ref_budget_s / max(1, args.steps + args.warmup)
    rows = int(max(1, min(units, budget / t_unit))) * gs
    for s in range(args.warmup):
        step(rows, s)
    t0 = time.perf_counter()
    for s in range(args.steps):
        step(rows, s)
    dt = time.perf_counter() - t0
    bytes_per_step = threads * ((rows // 2) * N + (rows // gs) * N * 3 + rows + N * 2)
    value = args.steps * bytes_per_step / dt / 1e9
    sample = (f"each step: {threads} threads each run the reference INT4 kernel on a {rows}-row K slice "
              f"at full N={N} (int8 activations, its only activation type); {args.steps} steps in {dt:.1f} s")
    line = {
        "metric": METRIC, "value": round(value, 4), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": dt * 1e3 / args.steps, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": WORKLOAD, "K": K, "N": N, "group_size": gs},
        "impl": "reference",
        "cpu_baseline": {"value": round(value, 4), "unit": "GB/s", "cores": threads, "kind": kind,
                         "sample": sample},
        "e2e": {"value": round(value, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


INT8_WORKLOAD = (f"int8_gemv: x fp32 [1,{K_DIM}] x W[{K_DIM}x{N_DIM}] int8 per-channel (fp32 column scales), "
                 f"y fp32 [1,{N_DIM}] (weight-only variant of the gemm_int8 shader, vulkan_shaders.h:53-82)")


def run_int8(args):
    """The INT8 per-channel decode GEMV (row a3): same timing rules as the INT4
    line; the reference has no CPU kernel for this layout (its only INT8 path
    is a GLSL/OpenCL shader), so there is no CPU baseline on this line."""
    import torch

    from silicongraph_b200 import _lib, kernels

    rank, local_rank, world = rank_env()
    if world > 1:
        raise SystemExit("--workload gemv_int8 runs on one GPU")
    torch.cuda.set_device(local_rank)
    lib = _lib.load()
    dev = torch.device("cuda", local_rank)
    K, N = K_DIM, N_DIM
    nbytes = K * N + 4 * N + 4 * K + 4 * N
    rng = np.random.default_rng(4321)
    W = (rng.standard_normal((K, N)) * 0.02).astype(np.float32)
    sc = (np.abs(W).max(axis=0) / 127.0).astype(np.float32)
    Wq = np.clip(np.rint(W / sc), -127, 127).astype(np.int8)
    l2 = torch.cuda.get_device_properties(dev).L2_cache_size
    copies = max(2, math.ceil(2.0 * l2 / (K * N)))
    Bs = [torch.from_numpy(Wq).to(dev) for _ in range(copies)]
    S = torch.from_numpy(sc).to(dev)
    x = torch.from_numpy(rng.standard_normal((1, K)).astype(np.float32)).to(dev)
    y = torch.empty((1, N), dtype=torch.float32, device=dev)
    params = [kernels.matmul_params(x, Bs[i], y, M=1, K=K, N=N, scales=S) for i in range(copies)]
    pptr = [ctypes.byref(p) for p in params]
    stream = torch.cuda.Stream(dev)
    st = stream.cuda_stream
    fn = lib.sg_matmul_int8_channel

    def launch(i):
        r = fn(pptr[i % copies], st)
        if r != 0:
            raise _lib.SgError(r, _lib.last_error())

    for i in range(args.warmup):
        launch(i)
    stream.synchronize()
    graph_len = max(copies, (min(args.graph_len, args.steps) // copies) * copies)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        for i in range(graph_len):
            launch(i)
    g.replay()
    stream.synchronize()
    clocks = ClockSampler(torch.cuda.current_device())
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        torch.cuda._sleep(2_000_000)  # host queues the launches while the GPU waits (outside the timed region)
        e0.record(stream)
        for _ in range(args.steps // graph_len):
            g.replay()
        for i in range(args.steps % graph_len):
            launch(i)
        e1.record(stream)
    stream.synchronize()
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = e0.elapsed_time(e1)
    value = args.steps * nbytes / (ms / 1e3) / 1e9
    peak, peak_src = read_peak_hbm()
    line = {
        "metric": "INT8 per-channel GEMV HBM GB/s", "value": round(value, 2), "unit": "GB/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded N(0,1) activations, N(0,0.02) weights quantised per column on the host)",
        "config": {"workload": INT8_WORKLOAD, "weight_copies": copies,
                   "l2": f"{copies} weight copies rotate ({copies * K * N / 1e6:.0f} MB > L2)"},
        "roofline": {"bound": "hbm", "achieved": round(value, 2), "peak": peak, "unit": "GB/s",
                     "frac": round(value / peak, 4), "peak_source": f"{peak_src} hbm_gbs", "traffic": None,
                     "achieved_basis": "algorithmic bytes per launch x launches / event time of back-to-back launches"},
        "cpu_baseline": None,
        "gpu_launches": args.steps,
        "clocks": clk,
    }
    return line


# Sub-results of the default run, measured in the same process after the
# headline: (name, workload, batch, steps, warmup).  One GPU: the other
# kernels of the hot path and the Llama-3.2-1B-shape decode; several GPUs: the
# same decode tensor-parallel over all of them (NCCL all-reduce after the
# row-parallel projections).
SUB_ONE_GPU = [
    ("gemv_int8", "gemv_int8", 1, 2000, 50),
    ("prefill_int4", "prefill_int4", 1, 10, 3),
    ("attn_prefill", "attn_prefill", 1, 10, 3),
    ("attn_small", "attn_small", 1, 20, 3),
    ("decode_llama1b_b1", "decode_llama1b", 1, 96, 4),
    ("decode_llama1b_b16", "decode_llama1b", 16, 96, 4),
]
SUB_MULTI_GPU = [
    ("decode_llama1b_tp_b1", "decode_llama1b_tp", 1, 96, 4),
    ("decode_llama1b_tp_b16", "decode_llama1b_tp", 16, 96, 4),
]
SUB_KEYS = ("metric", "value", "unit", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling", "dtype",
            "config", "roofline", "e2e", "cpu_baseline", "gpu_launches", "clocks")


def run_workload(args):
    if args.workload == "gemv_int8":
        return run_int8(args)
    if args.workload in PF_WORKLOADS:
        return run_prefill(args)
    if args.workload in ATTN_WORKLOADS:
        return run_attention(args)
    if args.workload in ("decode_llama1b", "decode_llama1b_tp"):
        return run_decode(args)
    if args.workload == "qwen7b_tp":
        return run_qwen(args)
    return run_ours(args)


def run_default(args):
    """The headline INT4 GEMV line with the sub-results in "sub_results"."""
    line = run_ours(args)
    if args.no_sub:
        return line
    _, _, world = rank_env()
    subs = {}
    for name, workload, batch, steps, warmup in (SUB_ONE_GPU if world == 1 else SUB_MULTI_GPU):
        ns = argparse.Namespace(**vars(args))
        ns.workload, ns.batch, ns.steps, ns.warmup = workload, batch, steps, warmup
        ns.cpu_seconds = min(args.cpu_seconds, 6.0)
        t0 = time.perf_counter()
        try:
            r = run_workload(ns)
            sub = {k: r[k] for k in SUB_KEYS if k in r}
        except Exception as e:  # a failing sub-result is reported, the headline stands
            sub = {"error": f"{type(e).__name__}: {str(e)[:300]}"}
        sub["wall_s"] = round(time.perf_counter() - t0, 1)
        subs[name] = sub
    line["sub_results"] = subs
    return line


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100000)
    ap.add_argument("--warmup", type=int, default=1000)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--graph-len", type=int, default=256)
    ap.add_argument("--e2e-steps", type=int, default=5000)
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--ref-budget-s", type=float, default=120.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-sub", action="store_true", help="default workload: the headline line only")
    ap.add_argument("--batch", type=int, default=1,
                    help="decode workloads: sequences decoded in lockstep by one session (config: 1 and 16)")
    ap.add_argument("--workload", choices=["gemv_int4", "gemv_int8", *PF_WORKLOADS, *ATTN_WORKLOADS, "decode_llama1b",
                                           "decode_llama1b_tp", "qwen7b_tp"],
                    default="gemv_int4",
                    help="gemv_int4 (default): the decode GEMV (columns split over the GPUs), with the other "
                         "workloads as sub-results; gemv_int8: the INT8 per-channel GEMV; prefill_int4 / "
                         "prefill_int8: the prefill GEMM; attn_prefill / attn_small: flash attention; "
                         "decode_llama1b: Llama-1B-shape decode through the SDK (one session per GPU); "
                         "decode_llama1b_tp: the same model tensor-parallel over all GPUs; qwen7b_tp: "
                         "Qwen-7B-shape 8192-token prefill + decode, tensor-parallel over all GPUs")
    ap.add_argument("--tuning", action="append", default=[], metavar="KEY=VALUE",
                    help="kernel tuning knob (sg_set_tuning) applied before the run; repeatable")
    args = ap.parse_args()
    if args.tuning:
        from silicongraph_b200 import kernels
        for kv in args.tuning:
            key, _, val = kv.partition("=")
            kernels.set_tuning(key, int(val))
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    rank, _, world = rank_env()
    if world != args.gpus and args.impl == "ours":
        if args.gpus > 1 and world == 1:
            ap.error("for --gpus N > 1 launch with torch.distributed.run --nproc-per-node N")
    if args.impl == "reference":
        if args.workload != "gemv_int4":
            ap.error("--impl reference times the decode GEMV workload")
        run_reference(args)
        return
    try:
        line = run_default(args) if args.workload == "gemv_int4" else run_workload(args)
        if rank == 0:
            print(json.dumps(line), flush=True)
    finally:
        dist_teardown()


if __name__ == "__main__":
    main()
