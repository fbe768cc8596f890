"""Benchmark of the B200 GEMM backend; prints ONE JSON line on rank 0.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
                    [--workload square8192|rowshard32768] [--quick]

Metric: device-timed TFLOP/s = 2*M*K*N / t (the reference's src/main.py:102).

* N = 1 (default workload ``square8192``): C = A*B with M=K=N=8192, BF16 inputs
  drawn N(0, 1/sqrt(K)) from a fixed seed, FP32 accumulate and output, through
  the library's C-ABI (``matmul_launch``, tcgen05 kernel), timed the reference's
  way (src/benchmark_backends.py:49-69): a step is one replay of a CUDA graph of
  10 GEMMs between external events, captured after 10 eager warm-up GEMMs; W
  untimed steps, then K timed steps (default 21); value = 2MKN / (median step /
  10).  A and B (134 MB each) and C (268 MB) are larger than the 126 MB L2, so
  no flush is needed between steps.  Extra fields: a back-to-back burst of the
  same launch, the same statistic for every precision beside torch/cuBLAS on the
  same inputs (replays alternating), the roofline, the CPU baseline and the
  end-to-end figure through the public API with host buffers.
* N > 1 (default workload ``rowshard32768``): M=K=N=32768 BF16, U[-1,1), A and C
  row-sharded over the ranks; every step broadcasts one B from rank 0 (posted
  one step ahead, overlapping the GEMMs: by copy engines over symmetric memory,
  ``--broadcast ce``, the default, or by NCCL on its own communicator) and
  gathers C on rank 0 (``--gather root``, the default: the single-GPU call's
  result, on one device) or on every rank (``--gather all``) in row chunks that
  overlap the next chunk's GEMM, with ``--reserve-sms`` SMs left to the NCCL
  kernels (2 with the copy-engine broadcast, 8 with NCCL's); one process per
  GPU under torchrun; time = max over ranks.  The other gather variant, each
  part of a step alone and T1 are timed in the same run.
* ``--impl reference`` times the reference's CPU path (numpy FP32 GEMM,
  src/benchmark_backends.py:223-226) on the host cores over row slabs of the
  same workload; under torchrun only rank 0 runs it.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
PACKAGE = ROOT / "matrix-multiplication_b200"
ORACLE = ROOT / "oracle"
sys.path.insert(0, str(PACKAGE))

METRIC = "device-timed TFLOP/s (2MKN/s) per precision at 4096³/8192³, % of B200 peak; 1/2/4/8-GPU"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "sm_max_mhz": 1965.0}
SM_COUNT = 148
FFMA_PER_SM_PER_CLK = 128


def load_peaks() -> tuple[dict, str]:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        try:
            return json.loads(path.read_text()), "measured"
        except ValueError:
            pass
    return dict(FALLBACK_PEAKS), "fallback"


def tflops(m, k, n, ms):
    return 2.0 * m * k * n / (ms * 1e-3) / 1e12


# ---------------------------------------------------------------- clocks
class ClockSampler:
    """SM clock, power and clock-event reasons of one GPU, sampled every `period`
    seconds on a background thread through NVML (nvidia-smi's -lms loop when NVML
    cannot be used); ``summary(t0, t1)`` keeps the samples taken in [t0, t1]."""

    REASON_BITS = {"hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40,
                   "sw_power_cap": 0x4, "hw_power_brake_slowdown": 0x80}
    SMI_FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
                  "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                  "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, cuda_index: int, period: float = 0.01):
        self.cuda_index = cuda_index
        self.period = period
        self.samples = []          # (time, sm_mhz, max_mhz, power_w, set of reasons)
        self.source = None
        self._stop = threading.Event()
        self._thread = None
        self._proc = None

    def _nvml_handle(self):
        import pynvml
        import torch

        pynvml.nvmlInit()
        try:
            uuid = str(torch.cuda.get_device_properties(self.cuda_index).uuid)
            return pynvml, pynvml.nvmlDeviceGetHandleByUUID(("GPU-" + uuid).encode())
        except Exception:
            visible = os.environ.get("CUDA_VISIBLE_DEVICES", "")
            ids = [v.strip() for v in visible.split(",") if v.strip()]
            index = int(ids[self.cuda_index]) if ids and ids[self.cuda_index].isdigit() else self.cuda_index
            return pynvml, pynvml.nvmlDeviceGetHandleByIndex(index)

    def _poll_nvml(self, nvml, handle):
        max_mhz = float(nvml.nvmlDeviceGetMaxClockInfo(handle, nvml.NVML_CLOCK_SM))
        while not self._stop.is_set():
            try:
                mhz = float(nvml.nvmlDeviceGetClockInfo(handle, nvml.NVML_CLOCK_SM))
                power = nvml.nvmlDeviceGetPowerUsage(handle) / 1000.0
                bits = nvml.nvmlDeviceGetCurrentClocksEventReasons(handle)
                reasons = {name for name, bit in self.REASON_BITS.items() if bits & bit}
                self.samples.append((time.time(), mhz, max_mhz, power, reasons))
            except Exception:
                pass
            self._stop.wait(self.period)

    def _poll_smi(self):
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for line in self._proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                reasons = {name for name, value in zip(names, parts[5:9]) if value.lower() == "active"}
                self.samples.append((time.time(), float(parts[1]), float(parts[2]), float(parts[3]), reasons))
            except ValueError:
                continue

    def __enter__(self):
        try:
            nvml, handle = self._nvml_handle()
            self.source = "nvml"
            self._thread = threading.Thread(target=self._poll_nvml, args=(nvml, handle), daemon=True)
        except Exception:
            try:
                self._proc = subprocess.Popen(
                    ["nvidia-smi", f"--query-gpu={self.SMI_FIELDS}", "--format=csv,noheader,nounits",
                     "-lms", str(max(10, int(self.period * 1000))), "-i", str(self.cuda_index)],
                    stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            except OSError:
                return self
            self.source = "nvidia-smi"
            self._thread = threading.Thread(target=self._poll_smi, daemon=True)
        self._thread.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._proc is not None:
            self._proc.terminate()
            try:
                self._proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self._proc.kill()
        if self._thread is not None:
            self._thread.join(timeout=5)

    def summary(self, start: float, stop: float) -> dict:
        rows = [row for row in self.samples if start <= row[0] <= stop]
        window = "timed region"
        if not rows:
            rows = list(self.samples)
            window = "whole run"
        mhz = [row[1] for row in rows]
        reasons = set().union(*(row[4] for row in rows)) if rows else set()
        return {"sm_mhz": statistics.median(mhz) if mhz else None,
                "sm_max_mhz": rows[-1][2] if rows else None,
                "power_w_max": max(row[3] for row in rows) if rows else None,
                "reasons": sorted(reasons), "samples": len(rows), "window": window,
                "window_s": stop - start, "source": self.source}


# ---------------------------------------------------------------- reference (CPU) arm
def run_reference_arm(args, rank: int) -> None:
    if rank != 0:
        return
    sys.path.insert(0, str(ORACLE))
    import numpy as np

    import cpu_backend

    m = k = n = 8192 if args.workload == "square8192" else 32768
    rows = 512
    rng = np.random.default_rng(2026)
    # The reference's CPU path is FP32 only: BF16-representable FP32 inputs.
    scale = np.float32(k ** -0.5) if args.workload == "square8192" else np.float32(1.0)
    a = (rng.standard_normal((rows * 2, k), dtype=np.float32) * scale)
    b = (rng.standard_normal((k, n), dtype=np.float32) * scale)
    out = np.empty((rows, n), dtype=np.float32)
    for i in range(args.warmup):
        cpu_backend.numpy_gemm(a[:rows], b, out)
    times = []
    for i in range(args.steps):
        start = time.perf_counter()
        cpu_backend.numpy_gemm(a[(i % 2) * rows:(i % 2 + 1) * rows], b, out)
        times.append(time.perf_counter() - start)
    total = sum(times)
    value = 2.0 * rows * k * n * args.steps / total / 1e12
    cores = cpu_backend.blas_threads()
    sample = f"{rows} x {k} @ {k} x {n} FP32 numpy row slab per step of the {m}x{k}x{n} workload"
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": total / args.steps * 1e3,
        "higher_is_better": True, "scaling": "strong" if args.gpus > 1 else "weak", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic (seeded normal, FP32)",
        "config": {"workload": f"{args.workload} (CPU row slabs)", "m": m, "k": k, "n": n,
                   "path": "numpy.matmul FP32 (src/benchmark_backends.py:223-226)"},
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": cores, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def cpu_baseline(seconds: float = 10.0) -> dict:
    sys.path.insert(0, str(ORACLE))
    import numpy as np

    import cpu_backend

    k = n = 8192
    rng = np.random.default_rng(2026)
    a = rng.standard_normal((1024, k), dtype=np.float32) * np.float32(k ** -0.5)
    b = rng.standard_normal((k, n), dtype=np.float32) * np.float32(k ** -0.5)
    result = cpu_backend.time_numpy_slabs(a, b, rows=512, seconds=seconds)
    return {"value": result["flops"] / result["seconds"] / 1e12, "unit": "TFLOP/s",
            "cores": cpu_backend.blas_threads(), "kind": "port",
            "sample": (f"{result['slabs']} row slabs of 512 x 8192 @ 8192 x 8192 FP32 numpy.matmul "
                       f"({result['seconds']:.1f} s) standing in for the 8192^3 GEMM")}


# ---------------------------------------------------------------- single GPU
def capture_graph_timer(call, stream, warmup=10):
    """One graph of DEVICE_BATCH calls between external events, after `warmup`
    eager calls: the capture half of the reference's measure_cuda_device
    (src/benchmark_backends.py:49-69)."""
    import torch
    from benchmark_backends import DEVICE_BATCH

    with torch.cuda.stream(stream):
        for _ in range(warmup):
            call()
    stream.synchronize()
    start = torch.cuda.Event(enable_timing=True, external=True)
    end = torch.cuda.Event(enable_timing=True, external=True)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        start.record(stream)
        for _ in range(DEVICE_BATCH):
            call()
        end.record(stream)
    graph.replay()
    end.synchronize()
    return graph, start, end


def interleaved_reference_method(timers, m, k, n, repeats=21) -> list[dict]:
    """The reference's statistic (median of `repeats` graph replays of DEVICE_BATCH
    calls) for several captured timers, replayed in turn so that every arm sees
    the same power and clock history."""
    from benchmark_backends import DEVICE_BATCH

    samples = [[] for _ in timers]
    for _ in range(repeats):
        for arm, (graph, start, end) in enumerate(timers):
            graph.replay()
            end.synchronize()
            samples[arm].append(start.elapsed_time(end) / DEVICE_BATCH)
    out = []
    for arm_samples in samples:
        median = statistics.median(arm_samples)
        out.append({"median_ms": median, "tflops": tflops(m, k, n, median)})
    return out


def single_gpu(args) -> dict:
    import numpy as np
    import torch

    from gpumat import NativeMatmul
    from precision import INPUT_DTYPES

    peaks, peak_kind = load_peaks()
    m = k = n = 8192
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    native = NativeMatmul(device=0)
    plan = native.plan("tcgen05", 8192, 8192, 8192, precision="bf16")
    stream = torch.cuda.Stream(device=device)
    gen = torch.Generator(device=device)
    gen.manual_seed(2026)
    with torch.cuda.stream(stream):
        a32 = torch.randn((m, k), generator=gen, device=device) * (k ** -0.5)
        b32 = torch.randn((k, n), generator=gen, device=device) * (k ** -0.5)
        a = torch.empty((m, k), dtype=torch.bfloat16, device=device)
        b = torch.empty((k, n), dtype=torch.bfloat16, device=device)
        native.convert(a32, a, "bf16")
        native.convert(b32, b, "bf16")
        c = torch.empty((m, n), dtype=torch.float32, device=device)
        run = native.prepare("tcgen05", a, b, c, precision="bf16")
    stream.synchronize()

    # ---- contract timing, the reference's own statistic (src/benchmark_backends.py:49-69):
    # one CUDA graph holds DEVICE_BATCH GEMMs between two external events and is
    # captured after 10 eager warm-up calls; a step is one replay of that graph.  W
    # untimed replays, then K timed replays between a synchronize on both sides; each
    # step's device time is its event interval, and value = 2MKN / (median / batch).
    from benchmark_backends import DEVICE_BATCH

    graph, g_start, g_end = capture_graph_timer(run, stream, warmup=10)
    for _ in range(args.warmup):
        graph.replay()
    stream.synchronize()
    samples = []
    with ClockSampler(0) as clocks:
        time.sleep(0.05)
        torch.cuda.synchronize()
        wall0 = time.time()
        for _ in range(args.steps):
            graph.replay()
            g_end.synchronize()
            samples.append(g_start.elapsed_time(g_end))
        torch.cuda.synchronize()
        wall1 = time.time()
    ms_per_step = statistics.median(samples)
    kernel_ms = ms_per_step / DEVICE_BATCH
    value = tflops(m, k, n, kernel_ms)
    achieved = value
    clock_summary = clocks.summary(wall0, wall1)
    del graph

    # ---- the same kernel as a burst: back-to-back launches between two events (no graph).
    burst_launches = 100
    b0, b1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        b0.record(stream)
        for _ in range(burst_launches):
            run()
        b1.record(stream)
    stream.synchronize()
    burst_ms = b0.elapsed_time(b1) / burst_launches
    burst = {"launches": burst_launches, "mean_ms": burst_ms, "tflops": tflops(m, k, n, burst_ms),
             "timing": "back-to-back launches between two CUDA events on the launching stream"}
    status = native.device_status()

    # ---- correctness cross-check against torch/cuBLAS on the same inputs (not an oracle).
    with torch.cuda.stream(stream):
        ref = torch.mm(a, b, out_dtype=torch.float32)
    stream.synchronize()
    check = {"max_abs_diff_vs_torch_cublas": float((ref - c).abs().max().item()),
             "c_abs_max": float(c.abs().max().item()), "device_status": status}
    del ref

    # ---- end to end through the public API (end_to_end.HostMatmul): pinned FP32
    # host A, B -> device, on-device RNE conversion to BF16, GEMM in row chunks
    # whose C blocks go back while later A blocks are still arriving.
    from end_to_end import HostMatmul

    host_a = a32.cpu().pin_memory()
    host_b = b32.cpu().pin_memory()
    host_c = torch.empty((m, n), dtype=torch.float32).pin_memory()
    e2e_steps = max(3, min(args.steps, 10))
    host_gemm = HostMatmul(native, m, k, n, "bf16", chunks=8, tail_chunks=2)
    for _ in range(2):
        host_gemm(host_a, host_b, host_c)
    wall_e0 = time.perf_counter()
    for _ in range(e2e_steps):
        host_gemm(host_a, host_b, host_c)
    e2e_ms = (time.perf_counter() - wall_e0) * 1e3 / e2e_steps
    check["e2e_max_abs_diff_vs_device_path"] = float((host_c - c.cpu()).abs().max().item())
    # The link's own floor for this call: the same host-to-device bytes alone, and
    # the C copy back alone (pinned buffers, one copy stream, wall clock).
    link = {}
    for label, copies in (("h2d_only_ms", ((host_gemm.b32, host_b), (host_gemm.a32, host_a))),
                          ("d2h_only_ms", ((host_c, host_gemm.c),))):
        times = []
        for _ in range(3):
            t0 = time.perf_counter()
            with torch.cuda.stream(host_gemm.copy_in):
                for dst, src in copies:
                    dst.copy_(src, non_blocking=True)
            host_gemm.copy_in.synchronize()
            times.append((time.perf_counter() - t0) * 1e3)
        link[label] = min(times)
    e2e = {"value": tflops(m, k, n, e2e_ms), "unit": "TFLOP/s",
           "h2d_bytes_per_step": host_gemm.bytes_in, "d2h_bytes_per_step": host_gemm.bytes_out,
           "ms_per_step": e2e_ms, "steps": e2e_steps, "timing": "host wall clock per call (the call synchronizes)",
           "link_ms": link,
           "path": "HostMatmul: pinned FP32 host A,B -> H2D (B, then A in 8 row blocks, the last split in 2) -> matmul_convert "
                   "(RNE to BF16) -> matmul_launch per block -> D2H of each C block overlapping later H2D"}
    del host_a, host_b, host_c, host_gemm

    # ---- every precision by the reference's own timing method, plus torch/cuBLAS.
    per_precision = {}
    cublas = {}
    if not args.quick:
        from precision import torch_precision

        for backend, precision in (("tcgen05", "bf16"), ("tcgen05", "fp16"), ("tcgen05", "tf32"), ("ffma", "fp32")):
            dtype = getattr(torch, INPUT_DTYPES[precision])
            with torch.cuda.stream(stream):
                if precision == "bf16":
                    pa, pb = a, b
                else:
                    pa = torch.empty((m, k), dtype=dtype, device=device)
                    pb = torch.empty((k, n), dtype=dtype, device=device)
                    native.convert(a32, pa, precision)
                    native.convert(b32, pb, precision)
                prun = native.prepare(backend, pa, pb, c, precision=precision)
            ours_timer = capture_graph_timer(prun, stream)
            with torch_precision(torch, precision):
                if precision in ("fp16", "bf16"):
                    trun = lambda pa=pa, pb=pb: torch.mm(pa, pb, out_dtype=torch.float32, out=c)
                else:
                    trun = lambda pa=pa, pb=pb: torch.mm(pa, pb, out=c)
                theirs_timer = capture_graph_timer(trun, stream)
            # The reference's statistic for both arms, their graph replays alternating.
            ours, theirs = interleaved_reference_method([ours_timer, theirs_timer], m, k, n)
            per_precision[precision] = dict(backend=backend, **ours)
            cublas[precision] = theirs
            del pa, pb, prun, ours_timer, theirs_timer
        ffma_peak = SM_COUNT * FFMA_PER_SM_PER_CLK * 2 * peaks.get("sm_max_mhz", 1965.0) * 1e6 / 1e12
        per_precision["fp32"]["ffma_peak_tflops_at_max_clock"] = ffma_peak
        per_precision["fp32"]["frac_of_ffma_peak"] = per_precision["fp32"]["tflops"] / ffma_peak
        for precision in ("bf16", "fp16"):
            per_precision[precision]["frac_of_bf16_peak"] = per_precision[precision]["tflops"] / peaks["bf16_tflops"]
        per_precision["tf32"]["frac_of_half_bf16_peak"] = per_precision["tf32"]["tflops"] / (peaks["bf16_tflops"] / 2)
    native.close()

    traffic = None
    traffic_file = ROOT / "profiles" / "ncu_traffic.json"
    if traffic_file.exists():
        traffic = json.loads(traffic_file.read_text()).get(f"{plan['kernel']}_{plan['tile_m']}x{plan['tile_n']}_bf16_8192")
    # The timed region is K replays of 10 GEMMs back to back: when the clock record
    # shows the power cap, the kernel ran in the sustained regime and the sustained
    # cuBLAS figure is its denominator; otherwise the burst figure.
    sustained = "sw_power_cap" in (clock_summary.get("reasons") or []) and "bf16_tflops_sustained" in peaks
    peak = peaks["bf16_tflops_sustained"] if sustained else peaks["bf16_tflops"]
    peak_name = "bf16_tflops_sustained (cuBLAS 8192^3 back to back for 4 s)" if sustained else \
        "bf16_tflops (burst, cuBLAS 8192^3)"
    return {
        "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: A, B ~ N(0, 1/sqrt(K)) from a fixed seed, rounded to BF16 (RNE)",
        "config": {"workload": "gemm_bf16_8192x8192x8192", "m": m, "k": k, "n": n, "precision": "bf16",
                   "backend": "tcgen05 (matmul_launch impl 7)", "output": "FP32 row-major",
                   "step": f"one replay of a CUDA graph of {DEVICE_BATCH} GEMMs between external events "
                           "(the reference's measure_cuda_device); value = 2MKN / (median step / "
                           f"{DEVICE_BATCH}), after 10 eager warm-up GEMMs and W warm-up replays",
                   "gemms_per_step": DEVICE_BATCH,
                   "l2": "inputs larger than L2 (A, B 134 MB each, C 268 MB > 126 MB L2); no flush",
                   "parallelism": "single GPU"},
        "step_ms": {"median": ms_per_step, "min": min(samples), "max": max(samples),
                    "mean": statistics.mean(samples)},
        "burst": burst,
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                     "frac": achieved / peak, "traffic": traffic,
                     "peak_source": f"{peak_kind} {peak_name}",
                     "frac_of_burst_peak": achieved / peaks["bf16_tflops"],
                     "kernel": f"{plan['kernel']} {plan['tile_m']}x{plan['tile_n']} BF16", "kernel_ms": kernel_ms,
                     "kernel_ms_source": "median graph step / GEMMs per step (CUDA events on the launching stream)",
                     "algorithmic_flops_per_launch": 2.0 * m * k * n},
        "cpu_baseline": cpu_baseline(),
        "e2e": e2e,
        "gpu_launches": args.steps * DEVICE_BATCH,
        "clocks": clock_summary,
        "check": check,
        "per_precision": per_precision,
        "torch_cublas": cublas,
    }


# ---------------------------------------------------------------- multi GPU
def multi_gpu(args, rank: int, world: int, local_rank: int) -> dict | None:
    """Row-sharded 32768^3 BF16 GEMM over `world` ranks (one process per GPU).

    A step: broadcast of the next step's B, one step ahead (``--broadcast ce``:
    copy-engine pushes over symmetric memory, ``sharded.CopyEngineBroadcast``;
    ``nccl``: NCCL on its own communicator), the local rows' GEMMs in row chunks, and the C gather of every chunk
    as soon as it is done, to rank 0 (``--gather root``) or to every rank
    (``--gather all``) -- by copy-engine pushes into the peers' C (``--exchange
    ce``, no SM taken from the GEMM), by this library's push kernel (``push``) or
    by grouped NCCL send/recv (``nccl``).  Time per step = max over ranks of
    CUDA-event time.  The same run also measures, on every rank: the other
    gather variant, each part of a step alone (GEMMs, broadcast, exchange), T1
    (the whole problem on one GPU, all GPUs at once), an FP64 check of rows
    received from peers, and an end-to-end step from pinned FP32 host buffers.
    """
    import datetime

    import torch
    import torch.distributed as dist

    from gpumat import NativeMatmul
    from sharded import (BroadcastPipeline, CopyEngineBroadcast, CopyEngineGather, KernelPushGather, ShardPlan,
                         pipelined_step, pipelined_step_ce)

    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180), device_id=device)
    b_group = dist.new_group(list(range(world)))       # B broadcasts on their own communicator
    size = args.size or 32768
    m = k = n = size
    plan = ShardPlan(m, k, n, world, rank, chunks=args.chunks, gather="all")
    plan_root = ShardPlan(m, k, n, world, rank, chunks=args.chunks, gather="root")
    start, stop = plan.local_rows
    native = NativeMatmul(device=local_rank)
    stream = torch.cuda.current_stream(device)

    def shard_a(owner: int) -> torch.Tensor:
        rows = plan.rows[owner][1] - plan.rows[owner][0]
        gen = torch.Generator(device=device)
        gen.manual_seed(1000 + owner)
        a32 = torch.rand((rows, k), generator=gen, device=device) * 2 - 1
        out = torch.empty((rows, k), dtype=torch.bfloat16, device=device)
        native.convert(a32, out, "bf16")
        return out

    a = shard_a(rank)
    if args.broadcast == "ce":
        import torch.distributed._symmetric_memory as symm_mem

        # Both B buffers in symmetric memory: every rank maps every peer's copies.
        b = symm_mem.empty((k, n), dtype=torch.bfloat16, device=device)
        b_next = symm_mem.empty((k, n), dtype=torch.bfloat16, device=device)
        b_handles = [symm_mem.rendezvous(b, dist.group.WORLD), symm_mem.rendezvous(b_next, dist.group.WORLD)]
    else:
        b = torch.empty((k, n), dtype=torch.bfloat16, device=device)
    if rank == 0:
        gen = torch.Generator(device=device)
        gen.manual_seed(7)
        b32 = torch.rand((k, n), generator=gen, device=device) * 2 - 1
        native.convert(b32, b, "bf16")
        del b32
    use_ce = args.exchange in ("ce", "push")
    if use_ce:
        import torch.distributed._symmetric_memory as symm_mem

        c = symm_mem.empty((m, n), dtype=torch.float32, device=device)
        handle = symm_mem.rendezvous(c, dist.group.WORLD)
        if args.exchange == "ce":
            gather_all = CopyEngineGather(plan, c, handle=handle, streams=args.ce_streams)
            gather_root = CopyEngineGather(plan_root, c, handle=handle, streams=args.ce_streams)
        else:
            def push(src, dsts, nbytes, push_stream, ctas):
                native.peer_push(src, dsts, nbytes, stream=push_stream, ctas=ctas)

            gather_all = KernelPushGather(plan, c, push, handle=handle, ctas=args.push_ctas)
            gather_root = KernelPushGather(plan_root, c, push, handle=handle, ctas=args.push_ctas)
    else:
        c = torch.empty((m, n), dtype=torch.float32, device=device)
    dist.broadcast(b, src=0)                            # the first step's B, before the loop
    if args.broadcast == "ce":
        b_next.copy_(b)                                 # rank 0: the next step's B (the same matrix here)
        pipe = CopyEngineBroadcast(b, b_next, b_group, b_handles)
        del b_next
    else:
        pipe = BroadcastPipeline(b, b_group)
    del b
    sms = torch.cuda.get_device_properties(device).multi_processor_count
    gemm_sms = max(2, sms - args.reserve_sms) if args.reserve_sms else sms
    native.set_sm_limit(gemm_sms if gemm_sms < sms else 0)
    runs = {}

    def gemm(a_rows, b_full, c_rows):
        key = (a_rows.data_ptr(), b_full.data_ptr(), c_rows.data_ptr())
        if key not in runs:
            runs[key] = native.prepare("tcgen05", a_rows, b_full, c_rows, precision="bf16")
        runs[key]()

    def step_all():
        if use_ce:
            pipelined_step_ce(plan, a, pipe, gather_all, gemm)
        else:
            pipelined_step(plan, a, pipe, c, gemm)

    def step_root():
        if use_ce:
            pipelined_step_ce(plan_root, a, pipe, gather_root, gemm)
        else:
            pipelined_step(plan_root, a, pipe, c, gemm)

    def gemm_only():
        for lo, hi in plan.chunk_ranges[rank]:
            gemm(a[lo:hi], pipe.current, c[start + lo:start + hi])

    def broadcast_only():
        pipe.start()
        pipe.finish()

    def exchange_only(root: bool = False):
        if use_ce:
            gather = gather_root if root else gather_all
            for index in range(plan.chunk_count):
                event = torch.cuda.Event()
                event.record()
                gather.post(index, event)
            gather.finish()
        else:
            from sharded import exchange_chunk

            works = []
            for index in range(plan.chunk_count):
                works.extend(exchange_chunk(plan_root if root else plan, index, c))
            for work in works:
                work.wait()

    def timed(fn, steps: int, warmup: int, clocks=None) -> tuple[float, tuple[float, float]]:
        for _ in range(warmup):
            fn()
        dist.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        wall0 = time.time()
        e0.record(stream)
        for _ in range(steps):
            fn()
        e1.record(stream)
        torch.cuda.synchronize()
        wall1 = time.time()
        dist.barrier()
        ms = torch.tensor([e0.elapsed_time(e1) / steps], device=device, dtype=torch.float64)
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        return float(ms.item()), (wall0, wall1)

    step_main, step_other = (step_root, step_all) if args.gather == "root" else (step_all, step_root)
    with ClockSampler(local_rank) as clocks:
        ms_per_step, window = timed(step_main, args.steps, args.warmup)
    clock_summary = clocks.summary(*window)
    side_steps = max(3, min(args.steps, 10))
    breakdown = {} if args.quick else {
        ("all_gather_ms" if args.gather == "root" else "gather_to_rank0_ms"): timed(step_other, side_steps, 2)[0],
        "gemm_only_ms": timed(gemm_only, side_steps, 2)[0],
        "broadcast_only_ms": timed(broadcast_only, side_steps, 2)[0],
        "exchange_only_ms": timed(exchange_only, side_steps, 2)[0],
        "exchange_to_rank0_only_ms": timed(lambda: exchange_only(root=True), side_steps, 2)[0],
    }

    # Timeline of one step (after two untimed ones): per event, ms from the
    # step's start on each rank; rank 0's value and the largest over ranks.
    trace = None
    if use_ce:
        plan_main, gather_main = (plan_root, gather_root) if args.gather == "root" else (plan, gather_all)
        for _ in range(2):
            step_main()
        torch.cuda.synchronize()
        dist.barrier()
        marks = []
        pipelined_step_ce(plan_main, a, pipe, gather_main, gemm, marks=marks)
        torch.cuda.synchronize()
        offsets = torch.tensor([marks[0][1].elapsed_time(event) for _, event in marks], device=device,
                               dtype=torch.float64)
        everyone = [torch.empty_like(offsets) for _ in range(world)]
        dist.all_gather(everyone, offsets)
        table = torch.stack(everyone).cpu()
        trace = {"ms_from_step_start": {name: {"rank0": round(float(table[0, i]), 3),
                                               "max": round(float(table[:, i].max()), 3)}
                                        for i, (name, _) in enumerate(marks)},
                 "marks": "gemm<i>: chunk i's GEMM done; exchange: this rank's pushes done; broadcast: the "
                          + ("this rank's copy-engine pushes of the next B done (the B is whole on every rank "
                             "at the max over ranks)" if args.broadcast == "ce" else "next step's B arrived")
                          + "; end: the step's last operation on the compute stream"}

    # FP64 check of rows received from a peer (its A shard is regenerated here
    # from the same seed): the GEMM and the exchange together.  All-gather: each
    # rank checks 64 rows of the next rank's shard; gather to root: rank 0 checks
    # 64 rows of every other rank's shard.
    def check_rows(owners) -> list[float]:
        worst = [0.0, 0.0]
        for owner in owners:
            owner_lo = plan.rows[owner][0]
            band = min(64, plan.rows[owner][1] - owner_lo)
            a_owner = shard_a(owner)
            ratio, max_err = native.check_fp64(a_owner[:band], pipe.current, c[owner_lo:owner_lo + band], "bf16")
            del a_owner
            worst = [max(worst[0], ratio), max(worst[1], max_err)]
        return worst

    c.fill_(float("nan"))
    timed(step_all, 1, 0)
    check = torch.tensor(check_rows([(rank + 1) % world]), device=device, dtype=torch.float64)
    c.fill_(float("nan"))
    timed(step_root, 1, 0)
    root_check = torch.tensor(check_rows(range(1, world)) if rank == 0 else [0.0, 0.0], device=device,
                              dtype=torch.float64)
    check = torch.maximum(check, root_check)
    dist.all_reduce(check, op=dist.ReduceOp.MAX)

    # T1: the whole problem on one GPU, measured on every GPU at once (no SM limit).
    native.set_sm_limit(0)
    gen = torch.Generator(device=device)
    gen.manual_seed(2000)
    a_full32 = torch.rand((m, k), generator=gen, device=device) * 2 - 1
    a_full = torch.empty((m, k), dtype=torch.bfloat16, device=device)
    native.convert(a_full32, a_full, "bf16")
    del a_full32
    run_full = native.prepare("tcgen05", a_full, pipe.current, c, precision="bf16")
    t1_ms, _ = timed(run_full, 3, 1)
    t1_min = torch.tensor([t1_ms], device=device, dtype=torch.float64)
    del run_full, a_full
    native.set_sm_limit(gemm_sms if gemm_sms < sms else 0)

    # End to end (skipped with --quick): pinned FP32 host A shard (every rank) and B (rank 0) -> device,
    # RNE conversion, the sharded step, the step's result back to pinned host
    # memory (gather to root: the whole C from rank 0; all-gather: each rank's rows).
    c_result = (c if rank == 0 else None) if args.gather == "root" else c[start:stop]
    h2d = (stop - start) * k * 4 + (k * n * 4 if rank == 0 else 0)
    d2h = c_result.numel() * 4 if c_result is not None else 0
    e2e_ms = float("nan")
    if not args.quick:
        host_a = (torch.rand((stop - start, k), device=device) * 2 - 1).cpu().pin_memory()
        host_b = (torch.rand((k, n), device=device) * 2 - 1).cpu().pin_memory() if rank == 0 else None
        host_c = torch.empty(c_result.shape, dtype=torch.float32).pin_memory() if c_result is not None else None
        dev_a32 = torch.empty((stop - start, k), dtype=torch.float32, device=device)
        dev_b32 = torch.empty((k, n), dtype=torch.float32, device=device) if rank == 0 else None

        def e2e_step():
            dev_a32.copy_(host_a, non_blocking=True)
            native.convert(dev_a32, a, "bf16")
            if rank == 0:
                dev_b32.copy_(host_b, non_blocking=True)
                native.convert(dev_b32, pipe.pending, "bf16")
            step_main()
            if host_c is not None:
                host_c.copy_(c_result, non_blocking=True)

        e2e_ms = timed(e2e_step, 3, 1)[0]
        del host_a, host_b, host_c, dev_a32, dev_b32
    del c_result

    status = native.device_status()
    status_t = torch.tensor([status], device=device, dtype=torch.int64)
    dist.all_reduce(status_t, op=dist.ReduceOp.MAX)
    dist.all_reduce(t1_min, op=dist.ReduceOp.MIN)
    native.close()
    if use_ce:
        del gather_all, gather_root, handle
    del pipe
    if args.broadcast == "ce":
        del b_handles
    dist.barrier()
    dist.destroy_process_group()
    if rank != 0:
        return None
    value = tflops(m, k, n, ms_per_step)
    t1_value = tflops(m, k, n, t1_ms)
    return {
        "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic: U[-1,1) from fixed seeds, rounded to BF16",
        "config": {"workload": f"rowshard_bf16_{m}x{k}x{n}", "m": m, "k": k, "n": n, "precision": "bf16",
                   "parallelism": f"row-sharded A/C over {world} ranks; every step broadcasts one B ("
                                  + ("copy engines" if args.broadcast == "ce" else "NCCL, own communicator")
                                  + ", posted one step ahead and overlapping the GEMMs) and "
                                  + ("gathers C on rank 0" if args.gather == "root" else "all-gathers C")
                                  + f" in {plan.chunk_count} row chunks, each chunk's exchange overlapping the "
                                  f"next chunk's GEMM",
                   "gather": args.gather,
                   "broadcast": ("copy-engine pushes over symmetric memory: rank 0 sends part j of B to rank j+1, "
                                 "a one-element all-reduce, each owner forwards its part to the other ranks, a "
                                 "second all-reduce at the end of the step") if args.broadcast == "ce"
                                else "NCCL broadcast on its own communicator",
                   "exchange": ("copy-engine pushes into the peers' C (symmetric memory, one cudaMemcpyAsync "
                                f"per peer and chunk, peers rank+1, rank+2, ... on {args.ce_streams} copy "
                                "stream(s)), completed by a one-element NCCL all-reduce")
                   if args.exchange == "ce" else
                   (f"this library's push kernel (matmul_peer_push, {args.push_ctas or 16} CTAs on the SMs the "
                    "GEMM leaves free) storing each chunk into every peer's C over NVLink, completed by a "
                    "one-element NCCL all-reduce") if args.exchange == "push"
                   else "grouped NCCL send/recv of each chunk",
                   "chunks": plan.chunk_count, "gemm_sms": gemm_sms, "l2": "inputs larger than L2"},
        "t1": {"ms": t1_ms, "tflops": t1_value, "fastest_gpu_ms": float(t1_min.item()),
               "how": "the whole problem as one GEMM on each GPU at once, in the same run (max over GPUs)",
               "efficiency_vs_t1": t1_ms / (world * ms_per_step)},
        "breakdown_ms": breakdown,
        "trace": trace,
        "bound": {"ingress_bytes_per_step_rank1": 2 * k * n + 4 * (m - (plan.rows[1][1] - plan.rows[1][0])) * n,
                  "ingress_bytes_per_step_rank0": 4 * (m - (stop - start)) * n,
                  "note": "every rank but 0 must receive one B (BF16) and the other ranks' C rows (FP32) per "
                          "step; rank 0 only the C rows"},
        "e2e": {"value": tflops(m, k, n, e2e_ms), "unit": "TFLOP/s", "ms_per_step": e2e_ms,
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "path": "pinned FP32 host A shard (every rank) and B (rank 0) -> H2D -> matmul_convert (RNE) -> "
                        "sharded step -> D2H of the result (gather to root: the whole C from rank 0; all-gather: "
                        "each rank's own rows); byte counts are rank 0's, time the max over ranks"},
        "check": {"check_fp64_ratio_max": float(check[0].item()), "check_fp64_max_abs_err": float(check[1].item()),
                  "what": "after an all-gather step, 64 rows of the next rank's shard as received by each rank; "
                          "after a gather-to-root step, 64 rows of every other rank's shard on rank 0; "
                          "against an FP64 product (C filled with NaN before each step)"},
        "gpu_launches": args.steps * plan.chunk_count,
        "clocks": clock_summary, "device_status": int(status_t.item()),
    }


def parse_args(argv: list[str] | None = None) -> argparse.Namespace:
    """Command line -> arguments, with the defaults that depend on other flags resolved
    (``--reserve-sms``, ``--workload``, ``--steps``)."""
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=None,
                        help="timed steps (default 500 for square8192, 20 for rowshard32768)")
    parser.add_argument("--warmup", type=int, default=10)
    parser.add_argument("--impl", choices=("b200", "reference"), default="b200")
    parser.add_argument("--workload", choices=("square8192", "rowshard32768"), default=None)
    parser.add_argument("--size", type=int, default=None, help="override the sharded problem size")
    parser.add_argument("--chunks", type=int, default=8)
    parser.add_argument("--reserve-sms", type=int, default=None,
                        help="multi-GPU: SMs left free of GEMM CTAs for the NCCL kernels that overlap them "
                             "(default 2 with --broadcast ce, whose only kernels are one-element all-reduces; "
                             "8 with --broadcast nccl)")
    parser.add_argument("--exchange", choices=("ce", "push", "nccl"), default="ce",
                        help="multi-GPU C exchange: copy-engine pushes over symmetric memory, this library's "
                             "push kernel over symmetric memory, or NCCL send/recv")
    parser.add_argument("--push-ctas", type=int, default=16, help="CTAs of the push kernel (--exchange push)")
    parser.add_argument("--broadcast", choices=("nccl", "ce"), default="ce",
                        help="multi-GPU B broadcast: NCCL on its own communicator, or copy-engine pushes over "
                             "symmetric memory (rank 0 scatters B's parts, their owners forward them)")
    parser.add_argument("--gather", choices=("root", "all"), default="root",
                        help="multi-GPU: where C is assembled in the timed step -- on rank 0 (the single-GPU "
                             "call's result, on one device) or on every rank; the other variant is timed "
                             "in the same run")
    parser.add_argument("--ce-streams", type=int, default=1,
                        help="copy streams of the copy-engine exchange (peers visited rank+1, rank+2, ...)")
    parser.add_argument("--quick", action="store_true",
                        help="skip the per-precision and cuBLAS tables (one GPU) or the per-part breakdown and the "
                             "end-to-end step (several GPUs)")
    parser.add_argument("--sweep", choices=("square", "llm", "ragged", "all", "legacy"), default=None,
                        help="instead of the contract line, time every shape of a configuration "
                             "(reference graph method, one JSON line per case, torch/cuBLAS beside it); "
                             "'legacy' times the reference's own kernels (oracle/_ref/matmul.so) at "
                             "4096^3 and 8192^3 as comparison rows")
    parser.add_argument("--cases", nargs="+", default=None, metavar="MxKxN:PREC[:normal]",
                        help="like --sweep, for the listed shapes (inputs U[-1,1), or N(0, 1/sqrt(K)) with :normal)")
    args = parser.parse_args(argv)
    if args.warmup < 3:
        parser.error("at least 3 warm-up steps")
    if args.reserve_sms is None:
        args.reserve_sms = 2 if args.broadcast == "ce" else 8
    if args.workload is None:
        args.workload = "square8192" if args.gpus == 1 else "rowshard32768"
    if args.steps is None:
        args.steps = 21 if args.workload == "square8192" else 20
    args.parser = parser
    return args


def main() -> int:
    args = parse_args()
    parser = args.parser
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.sweep == "legacy":
        legacy_sweep()
        return 0
    if args.sweep or args.cases:
        sweep(args.sweep, [parse_case(text) for text in args.cases] if args.cases else None)
        return 0
    if args.impl == "reference":
        run_reference_arm(args, rank)
        return 0
    if world > 1 or args.workload == "rowshard32768":
        if world == 1 and args.gpus > 1:
            parser.error("--gpus > 1 needs torchrun with one process per GPU")
        line = multi_gpu(args, rank, world, local_rank) if world > 1 else None
        if world == 1:
            line = single_rowshard(args)
    else:
        line = single_gpu(args)
    if line is not None:
        print(json.dumps(line), flush=True)
    return 0


SWEEPS = {
    # square size sweep 64..4096 at every precision, U[-1,1)
    "square": [(s, s, s, p, "uniform") for s in (64, 128, 256, 512, 1024, 2048, 4096)
               for p in ("fp32", "tf32", "fp16", "bf16")],
    # large and LLM-like shapes, BF16 and FP16, N(0, 1/sqrt(K))
    "llm": [(m, k, n, p, "normal") for (m, k, n) in ((8192, 8192, 8192), (16, 8192, 8192),
                                                      (8192, 8192, 28672), (4096, 14336, 4096))
            for p in ("bf16", "fp16")],
    # ragged partial-tile shapes, FP32 and BF16
    "ragged": [(m, k, n, p, "uniform") for (m, k, n) in ((31, 33, 65), (511, 257, 129), (513, 129, 577))
               for p in ("fp32", "bf16")],
}


def parse_case(text: str) -> tuple:
    """``"MxKxN:prec"`` or ``"MxKxN:prec:normal"`` -> (m, k, n, prec, distribution)."""
    parts = text.split(":")
    if len(parts) not in (2, 3) or parts[1] not in ("fp32", "tf32", "fp16", "bf16") or \
            (len(parts) == 3 and parts[2] not in ("normal", "uniform")):
        raise SystemExit(f"bad case {text!r}: use MxKxN:fp32|tf32|fp16|bf16[:normal]")
    dims = parts[0].lower().split("x")
    if len(dims) != 3 or not all(d.isdigit() and int(d) > 0 for d in dims):
        raise SystemExit(f"bad case {text!r}: the shape is MxKxN with positive sizes")
    m, k, n = (int(d) for d in dims)
    return m, k, n, parts[1], parts[2] if len(parts) == 3 else "uniform"


def sweep(which: str | None, explicit: list | None = None) -> None:
    """Time each case with the reference's CUDA-graph method; print one JSON line per case."""
    import torch

    from gpumat import NativeMatmul
    from precision import INPUT_DTYPES, torch_precision

    peaks, _ = load_peaks()
    cases = explicit if explicit is not None else \
        [c for key in (("square", "llm", "ragged") if which == "all" else (which,)) for c in SWEEPS[key]]
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    native = NativeMatmul(device=0)
    stream = torch.cuda.Stream(device=device)
    for m, k, n, precision, dist in cases:
        backend = "ffma" if precision == "fp32" else "tcgen05"
        dtype = getattr(torch, INPUT_DTYPES[precision])
        gen = torch.Generator(device=device)
        gen.manual_seed(m * 7 + k * 3 + n)
        with torch.cuda.stream(stream):
            if dist == "normal":
                a32 = torch.randn((m, k), generator=gen, device=device) * (k ** -0.5)
                b32 = torch.randn((k, n), generator=gen, device=device) * (k ** -0.5)
            else:
                a32 = torch.rand((m, k), generator=gen, device=device) * 2 - 1
                b32 = torch.rand((k, n), generator=gen, device=device) * 2 - 1
            a = torch.empty((m, k), dtype=dtype, device=device)
            b = torch.empty((k, n), dtype=dtype, device=device)
            native.convert(a32, a, precision)
            native.convert(b32, b, precision)
            del a32, b32
            c = torch.empty((m, n), dtype=torch.float32, device=device)
            ref = torch.empty((m, n), dtype=torch.float32, device=device)
            run = native.prepare(backend, a, b, c, precision=precision)
        ours_timer = capture_graph_timer(run, stream)
        with torch_precision(torch, precision):
            if precision in ("fp16", "bf16"):
                trun = lambda: torch.mm(a, b, out_dtype=torch.float32, out=ref)
            else:
                trun = lambda: torch.mm(a, b, out=ref)
            theirs_timer = capture_graph_timer(trun, stream)
        ours, theirs = interleaved_reference_method([ours_timer, theirs_timer], m, k, n)
        del ours_timer, theirs_timer
        stream.synchronize()
        diff = float((c - ref).abs().max().item())
        with torch.cuda.stream(stream):
            check_ratio, check_err = native.check_fp64(a, b, c, precision)
        bytes_min = (4 if precision in ("fp32", "tf32") else 2) * (m * k + k * n) + 4 * m * n
        line = {"case": f"{m}x{k}x{n}", "precision": precision, "backend": backend,
                "median_ms": ours["median_ms"], "tflops": ours["tflops"],
                "gbs_min_bytes": bytes_min / (ours["median_ms"] * 1e-3) / 1e9,
                "frac_bf16_peak": ours["tflops"] / peaks["bf16_tflops"],
                "torch_cublas_tflops": theirs["tflops"], "ratio_vs_cublas": ours["tflops"] / theirs["tflops"],
                "max_abs_diff_vs_cublas": diff, "inputs": dist,
                "check_fp64_ratio": check_ratio, "check_fp64_max_abs_err": check_err,
                "check": "matmul_check_fp64 over every output (FP64 product of the rounded inputs, "
                         "the reference's GemmReference allowance; <= 1 passes)",
                "timing": "reference graph method (median of 21 replays of 10 GEMMs after 10 warmups), "
                          "replays alternating with cuBLAS's"}
        print(json.dumps(line), flush=True)
        del a, b, c, ref, run
    status = native.device_status()
    native.close()
    if status:
        raise RuntimeError(f"device status {status:#x}")


LEGACY_IMPLEMENTATIONS = {"fp32": ((2, "cublas"), (4, "warp_large"), (5, "pipeline")),
                          "tf32": ((2, "cublas"), (6, "wmma")), "fp16": ((2, "cublas"), (6, "wmma")),
                          "bf16": ((2, "cublas"), (6, "wmma"))}


def legacy_sweep(sizes=(4096, 8192)) -> None:
    """Comparison rows: the reference's own CUDA library (its src/matmul.cu built
    unmodified for sm_100a into oracle/_ref/matmul.so) -- its cuBLAS branch, its
    cp.async FP32 kernels and its wmma tensor-core kernel (src/matmul.cu:401-474)
    -- timed with the same graph method and inputs as this library, whose row is
    printed beside each.  These rows measure the reference's kernels, not this
    library; every output is checked by matmul_check_fp64."""
    import ctypes

    import torch

    from gpumat import NativeMatmul
    from precision import INPUT_DTYPES, torch_precision

    path = ROOT / "oracle" / "_ref" / "matmul.so"
    if not path.exists():
        print(json.dumps({"legacy": "unavailable", "why": f"{path} not built (make -C oracle ref)"}), flush=True)
        return
    ref = ctypes.CDLL(str(path))
    ref.matmul_create.restype = ctypes.c_void_p
    ref.matmul_create.argtypes = [ctypes.c_int, ctypes.c_char_p, ctypes.c_size_t]
    ref.matmul_destroy.argtypes = [ctypes.c_void_p, ctypes.c_char_p, ctypes.c_size_t]
    ref.matmul_launch.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p,
                                  ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p,
                                  ctypes.c_char_p, ctypes.c_size_t]
    err = ctypes.create_string_buffer(1024)
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    ref_ctx = ref.matmul_create(0, err, len(err))
    if not ref_ctx:
        raise RuntimeError(f"reference matmul_create failed: {err.value.decode()}")
    native = NativeMatmul(device=0)
    stream = torch.cuda.Stream(device=device)
    precision_ids = {"fp32": 0, "tf32": 1, "fp16": 2, "bf16": 3}
    for size in sizes:
        m = k = n = size
        for precision, impls in LEGACY_IMPLEMENTATIONS.items():
            dtype = getattr(torch, INPUT_DTYPES[precision])
            gen = torch.Generator(device=device)
            gen.manual_seed(size + len(precision))
            with torch.cuda.stream(stream):
                a32 = torch.rand((m, k), generator=gen, device=device) * 2 - 1
                b32 = torch.rand((k, n), generator=gen, device=device) * 2 - 1
                a = torch.empty((m, k), dtype=dtype, device=device)
                b = torch.empty((k, n), dtype=dtype, device=device)
                native.convert(a32, a, precision)
                native.convert(b32, b, precision)
                del a32, b32
                c = torch.empty((m, n), dtype=torch.float32, device=device)
                ours = native.prepare("ffma" if precision == "fp32" else "tcgen05", a, b, c, precision=precision)
            stream_ptr = ctypes.c_void_p(stream.cuda_stream)

            def legacy_call(impl):
                def call():
                    if ref.matmul_launch(ref_ctx, impl, precision_ids[precision], ctypes.c_void_p(a.data_ptr()),
                                         ctypes.c_void_p(b.data_ptr()), ctypes.c_void_p(c.data_ptr()), m, k, n,
                                         stream_ptr, err, len(err)) != 0:
                        raise RuntimeError(f"reference matmul_launch failed: {err.value.decode()}")
                return call

            timers = [capture_graph_timer(ours, stream)]
            names = ["b200 (this library)"]
            with torch_precision(torch, precision):
                for impl, name in impls:
                    timers.append(capture_graph_timer(legacy_call(impl), stream))
                    names.append(f"reference {name} (impl {impl})")
            results = interleaved_reference_method(timers, m, k, n)
            del timers
            for (impl_name, result), impl in zip(zip(names, results), [None] + [i for i, _ in impls]):
                with torch.cuda.stream(stream):
                    if impl is None:
                        ours()
                    else:
                        legacy_call(impl)()
                    ratio, max_err = native.check_fp64(a, b, c, precision)
                print(json.dumps({"case": f"{m}x{k}x{n}", "precision": precision, "implementation": impl_name,
                                  "median_ms": result["median_ms"], "tflops": result["tflops"],
                                  "check_fp64_ratio": ratio, "check_fp64_max_abs_err": max_err,
                                  "timing": "reference graph method (median of 21 replays of 10 GEMMs after 10 "
                                            "warmups), replays of all rows of the case alternating",
                                  "inputs": "U[-1,1) rounded to the input precision"}), flush=True)
            del a, b, c, ours
    status = native.device_status()
    native.close()
    ref.matmul_destroy(ref_ctx, err, len(err))
    if status:
        raise RuntimeError(f"device status {status:#x}")


def single_rowshard(args) -> dict:
    """The row-sharded workload on one GPU (its T1): one full GEMM per step."""
    import torch

    from gpumat import NativeMatmul

    size = args.size or 32768
    m = k = n = size
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    native = NativeMatmul(device=0)
    gen = torch.Generator(device=device)
    gen.manual_seed(1000)
    a32 = torch.rand((m, k), generator=gen, device=device) * 2 - 1
    a = torch.empty((m, k), dtype=torch.bfloat16, device=device)
    native.convert(a32, a, "bf16")
    del a32
    b32 = torch.rand((k, n), generator=gen, device=device) * 2 - 1
    b = torch.empty((k, n), dtype=torch.bfloat16, device=device)
    native.convert(b32, b, "bf16")
    del b32
    c = torch.empty((m, n), dtype=torch.float32, device=device)
    run = native.prepare("tcgen05", a, b, c, precision="bf16")
    for _ in range(args.warmup):
        run()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(0) as clocks:
        wall0 = time.time()
        e0.record()
        for _ in range(args.steps):
            run()
        e1.record()
        torch.cuda.synchronize()
        wall1 = time.time()
    ms_per_step = e0.elapsed_time(e1) / args.steps
    status = native.device_status()
    native.close()
    return {
        "metric": METRIC, "value": tflops(m, k, n, ms_per_step), "unit": "TFLOP/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: U[-1,1) from fixed seeds, rounded to BF16",
        "config": {"workload": f"rowshard_bf16_{m}x{k}x{n}", "m": m, "k": k, "n": n, "precision": "bf16",
                   "parallelism": "single GPU (T1 of the row-sharded workload)", "l2": "inputs larger than L2"},
        "gpu_launches": args.steps, "clocks": clocks.summary(wall0, wall1), "device_status": status,
    }


if __name__ == "__main__":
    raise SystemExit(main())
