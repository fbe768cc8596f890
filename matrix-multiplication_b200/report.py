"""``results.json`` (schema 3) and ``results.csv`` for the B200 backends.

The reference's benchmark driver (``src/main.py:199-279``) draws seeded
standard-normal FP32 inputs per shape, prepares every (backend, precision),
validates the device output and the end-to-end output against an FP64 reference
(``GemmReference.verify``, ``src/precision.py:134-161``), times each requested
mode, and writes ``results.json`` with ``schema_version`` 3 (``main.py:184-196,
236``) plus a CSV without the raw samples.  This module produces the same report
for this library's backends (``tcgen05``, ``ffma``) and for torch/cuBLAS
(``torch``) on one GPU, so the files drop into the reference's tooling:

* rows carry the reference's keys (``main.py:91-103``): backend, execution_device,
  precision, input_dtype, output_dtype, mode, m, k, n, median_ms, p10_ms, p90_ms,
  tflops, setup_ms, kernel_config, the error fields of ``GemmReference.verify``
  and samples_ms; ``kernel_config`` of the native backends is ``matmul_kernel_info``
  plus the per-shape ``matmul_plan``;
* modes: ``device`` (CUDA graph of 10 calls between events,
  ``benchmark_backends.measure_cuda_device``), ``resident`` and ``end_to_end``
  (synchronised wall time, ``main.py:77-88``);
* validation runs on the GPU in FP64 with torch (products of the precision-rounded
  inputs, the allowance atol + rtol*|ref| + gamma_K*(|A||B|) with u = 2^-23, the
  TF32 magnitude envelope and, for library TF32 only, the ties-away and unrounded
  candidate references), plus the library's own ``matmul_check_fp64`` ratio for
  the native backends; a failed check raises like the reference.

Plots are not produced (the reference's matplotlib output is out of scope).

Usage::

    python matrix-multiplication_b200/report.py --sizes 1024 4096 --precisions fp32 tf32 fp16 bf16 \\
        --modes device resident end_to_end --output results/
"""

from __future__ import annotations

import argparse
import csv
import hashlib
import json
import math
import platform
import statistics
import sys
import time
from pathlib import Path

HERE = Path(__file__).resolve().parent
if str(HERE) not in sys.path:
    sys.path.insert(0, str(HERE))

from precision import ATOL, BACKEND_PRECISIONS, INPUT_DTYPES, PRECISIONS, RTOL  # noqa: E402

SCHEMA_VERSION = 3
MODES = ("device", "resident", "end_to_end")
BACKENDS = ("tcgen05", "ffma", "torch")
TIMING = {
    "device": "CUDA graph events averaged over device_batch dispatches; no host transfers or Python enqueue gaps",
    "resident": "synchronized wall time with converted resident inputs and reused output; includes dispatch",
    "end_to_end": "wall time from original FP32 host inputs to owned FP32 host output; allocations, "
                  "placement, device-side conversion and readback included; the backend context is retained",
}


def parse_shape(text: str) -> tuple[int, int, int]:
    """``"M"`` (square) or ``"MxKxN"`` -> (m, k, n)."""
    parts = [int(p) for p in text.lower().replace("×", "x").split("x")]
    if len(parts) == 1:
        parts *= 3
    if len(parts) != 3 or min(parts) < 1:
        raise ValueError(f"bad shape {text!r}: use M or MxKxN with positive sizes")
    return parts[0], parts[1], parts[2]


def backend_supports(backend: str, precision: str) -> bool:
    return backend == "torch" or precision in BACKEND_PRECISIONS[backend]


def gamma(k: int, unit_roundoff: float) -> float:
    """gamma_K = K u / (1 - K u) (``precision.py:125-131``); infinite when K u >= 1."""
    ku = k * unit_roundoff
    return math.inf if ku >= 1 else ku / (1 - ku)


def result_row(backend, precision, mode, shape, samples, errors, setup_ms, execution_device, config) -> dict:
    """One measurement row with the reference's keys (``main.py:91-103``)."""
    m, k, n = shape
    if not samples or not all(math.isfinite(v) and v > 0 for v in samples):
        raise RuntimeError(f"{backend}/{mode}: invalid timing samples")
    ordered = sorted(samples)
    median = statistics.median(samples)
    return {"backend": backend, "execution_device": execution_device, "precision": precision,
            "input_dtype": INPUT_DTYPES[precision], "output_dtype": "float32", "mode": mode,
            "m": m, "k": k, "n": n, "median_ms": median, "p10_ms": _percentile(ordered, 10),
            "p90_ms": _percentile(ordered, 90), "tflops": 2 * m * k * n / (median * 1e9), "setup_ms": setup_ms,
            "kernel_config": config, **errors, "samples_ms": list(samples)}


def _percentile(ordered: list[float], q: float) -> float:
    """Linear-interpolation percentile (numpy's default method)."""
    position = (len(ordered) - 1) * q / 100.0
    low = math.floor(position)
    high = min(low + 1, len(ordered) - 1)
    return float(ordered[low] + (ordered[high] - ordered[low]) * (position - low))


def write_report(report: dict, output: Path) -> None:
    """results.json (indented, no NaN) and results.csv without samples (``main.py:184-196``); rows
    that lack a column (the native-only checker ratio) leave it empty."""
    output.mkdir(parents=True, exist_ok=True)
    (output / "results.json").write_text(json.dumps(report, indent=2, allow_nan=False) + "\n")
    rows = report["measurements"]
    if not rows:
        return
    columns = []
    for row in rows:                       # the union of row keys, in order of first appearance
        columns += [name for name in row if name != "samples_ms" and name not in columns]
    with (output / "results.csv").open("w", newline="") as file:
        writer = csv.DictWriter(file, fieldnames=columns)
        writer.writeheader()
        for row in rows:
            writer.writerow({key: json.dumps(row[key], sort_keys=True) if isinstance(row.get(key), dict)
                             else row.get(key) for key in columns})


def measure_wall(call, synchronize, warmup: int, repeats: int) -> list[float]:
    """Synchronised wall-clock samples in milliseconds (``main.py:77-88``)."""
    for _ in range(warmup):
        call()
        synchronize()
    samples = []
    for _ in range(repeats):
        synchronize()
        start = time.perf_counter_ns()
        call()
        synchronize()
        samples.append((time.perf_counter_ns() - start) / 1e6)
    return samples


class GpuReference:
    """FP64 references of one problem on the GPU (torch), mirroring ``GemmReference``."""

    def __init__(self, torch, native, a32, b32, precision: str):
        self.torch = torch
        self.precision = precision
        a64, b64 = a32.double(), b32.double()
        self.original = a64 @ b64
        left, right = self._rounded(native, a32), self._rounded(native, b32)
        self.rounded = self.original if precision == "fp32" else left @ right
        self.candidates = {"rounded_inputs": self.rounded}
        mag_left, mag_right = left.abs(), right.abs()
        if precision == "tf32":
            away_left, away_right = _ties_away_tf32(torch, a32), _ties_away_tf32(torch, b32)
            self.candidates["tf32_ties_away"] = away_left @ away_right
            self.candidates["original_fp32"] = self.original
            mag_left = torch.maximum(torch.maximum(mag_left, away_left.abs()), a64.abs())
            mag_right = torch.maximum(torch.maximum(mag_right, away_right.abs()), b64.abs())
        unit = 2.0 ** -23
        self.bound = gamma(a32.shape[1], unit) * (mag_left @ mag_right)

    def _rounded(self, native, x32):
        torch = self.torch
        if self.precision == "fp32":
            return x32.double()
        dst = torch.empty_like(x32, dtype=getattr(torch, INPUT_DTYPES[self.precision]))
        native.convert(x32.contiguous(), dst, self.precision)
        return dst.double()

    def verify(self, actual, label: str, *, allow_tf32_library: bool = False) -> dict:
        torch = self.torch
        if not torch.isfinite(actual).all():
            raise RuntimeError(f"{label}: expected finite FP32 output")
        result = actual.double()
        names = list(self.candidates) if (allow_tf32_library and self.precision == "tf32") else ["rounded_inputs"]
        best = None
        for name in names:
            reference = self.candidates[name]
            allowance = ATOL + RTOL * reference.abs() + self.bound
            scaled = float(((result - reference).abs() / allowance).max())
            if best is None or scaled < best[0]:
                best = (scaled, name, reference)
        scaled, name, reference = best
        if scaled > 1:
            raise RuntimeError(f"{label}: incorrect GEMM (roundoff-aware tolerance ratio {scaled:.3g})")

        def relative(diff, ref):
            norm = float(torch.linalg.vector_norm(ref))
            return None if norm == 0 else float(torch.linalg.vector_norm(diff)) / norm

        return {
            "max_abs_error": float((result - self.original).abs().max()),
            "arithmetic_max_abs_error": float((result - reference).abs().max()),
            "max_tolerance_ratio": scaled,
            "arithmetic_reference": name,
            "roundoff_bound_max": float(self.bound.max()),
            "relative_frobenius_error": relative(result - self.original, self.original),
            "arithmetic_relative_error": relative(result - reference, reference),
            "quantization_relative_error": relative(reference - self.original, self.original),
        }


def _ties_away_tf32(torch, x32):
    """TF32 rounding with ties away from zero (the library model of ``precision.py:66-76``)."""
    bits = x32.contiguous().view(torch.int32)
    finite = (bits & 0x7F800000) != 0x7F800000
    rounded = torch.where(finite, (bits + 0x1000) & ~0x1FFF, bits)
    return rounded.view(torch.float32).double()


def _file_digest(path: Path) -> str:
    with path.open("rb") as file:
        return hashlib.file_digest(file, "sha256").hexdigest()


def run(args) -> dict:
    import numpy as np
    import torch

    from benchmark_backends import DEVICE_BATCH, cuda_case, measure_cuda_device
    from gpumat import NativeMatmul
    from precision import torch_precision

    device = torch.device("cuda", args.device)
    torch.cuda.set_device(device)
    start = time.perf_counter_ns()
    native = NativeMatmul(args.library, device=args.device)
    init_ms = (time.perf_counter_ns() - start) / 1e6
    props = torch.cuda.get_device_properties(device)
    metadata = {
        "python": sys.version, "platform": platform.platform(), "machine": platform.machine(), "target": "cuda",
        "cpu": platform.processor(), "numpy": np.__version__, "cpu_threads": args.cpu_threads,
        "blas": np.show_config(mode="dicts"), "precisions": args.precisions,
        "input_dtypes": {p: INPUT_DTYPES[p] for p in args.precisions}, "output_dtype": "float32",
        "rounding": "FP16/BF16/TF32 inputs rounded to nearest even; library (torch) TF32 may use ties-away or FP32",
        "reduced_precision_reduction": False,
        "reference": "FP64 (GPU) of precision-rounded inputs; total error separately uses original FP32 inputs",
        "tf32_policy": "tcgen05 TF32 uses RNE; torch/cuBLAS validation accepts RNE, ties-away or IEEE FP32",
        "rtol": RTOL, "atol": ATOL, "seed": args.seed, "warmup": args.warmup, "repeats": args.repeats,
        "arithmetic_bound": "atol + rtol*abs(reference) + gamma_K*(abs(A)@abs(B)); FP32 u=2^-23; "
                            "TF32 uses upper envelope of legal inputs",
        "shapes_mkn": [list(s) for s in args.shapes], "backends": args.backends, "modes": args.modes,
        "device_batch": DEVICE_BATCH, "timing": TIMING,
        "cuda": torch.version.cuda, "torch": torch.__version__,
        "gpu": {"name": props.name, "capability": list(torch.cuda.get_device_capability(device)),
                "multiprocessors": props.multi_processor_count, "memory_bytes": props.total_memory},
        "native_libraries": {"b200_matmul": {"path": str(native.path), "sha256": _file_digest(native.path),
                                             "abi": 3}},
        "backend_initialization_ms": {"cuda": init_ms},
    }
    unsupported = [{"backend": b, "precision": p, "mode": m, "reason": f"{b} has no {p} kernel"}
                   for b in args.backends for p in args.precisions for m in args.modes if not backend_supports(b, p)]
    report = {"schema_version": SCHEMA_VERSION, "metadata": metadata, "measurements": [],
              "unsupported_cases": unsupported}
    stream = torch.cuda.Stream(device=device)
    rng = np.random.default_rng(args.seed)
    for shape in args.shapes:
        m, k, n = shape
        a = rng.standard_normal((m, k), dtype=np.float32)
        b = rng.standard_normal((k, n), dtype=np.float32)
        a32 = torch.from_numpy(a).to(device)
        b32 = torch.from_numpy(b).to(device)
        for precision in args.precisions:
            reference = GpuReference(torch, native, a32, b32, precision)
            for backend in args.backends:
                if not backend_supports(backend, precision):
                    continue
                label = f"{backend}/{precision} {m}x{k}x{n}"
                with torch_precision(torch, precision):
                    t0 = time.perf_counter_ns()
                    if backend == "torch":
                        case = _torch_case(torch, a, b, precision, stream, device)
                    else:
                        case = cuda_case(native, backend, precision, a, b, stream)
                    case.run()
                    case.synchronize()
                    setup_ms = (time.perf_counter_ns() - t0) / 1e6
                    library = backend == "torch"
                    out = torch.from_numpy(case.output()).to(device)
                    errors = reference.verify(out, label, allow_tf32_library=library)
                    reference.verify(torch.from_numpy(case.end_to_end()).to(device), label + "/end_to_end",
                                     allow_tf32_library=library)
                    config = case.config
                    if not library:
                        dtype = getattr(torch, INPUT_DTYPES[precision])
                        ratio, _ = native.check_fp64(a32.to(dtype), b32.to(dtype), out, precision)
                        errors["gpu_checker_tolerance_ratio"] = ratio
                        config = dict(config or {}, plan=native.plan(backend, m, k, n, precision=precision))
                    for mode in args.modes:
                        if mode == "device":
                            samples = measure_cuda_device(case.run, stream, args.warmup, args.repeats)
                        else:
                            call = case.run if mode == "resident" else case.end_to_end
                            samples = measure_wall(call, case.synchronize, args.warmup, args.repeats)
                        row = result_row(backend, precision, mode, shape, samples, errors, setup_ms,
                                         case.execution_device, config)
                        report["measurements"].append(row)
                        print(f"{backend:<8} {precision:<5} {m}x{k}x{n:<10} {mode:<11} {row['median_ms']:10.4f} ms "
                              f"{row['tflops']:9.3f} TFLOP/s  ratio {errors['max_tolerance_ratio']:.3f}", flush=True)
                del case
        del a32, b32
    status = native.device_status()
    if status:
        raise RuntimeError(f"device status {status:#x}")
    native.close()
    return report


def _torch_case(torch, a, b, precision, stream, device):
    """torch.matmul (cuBLAS) on resident inputs of the input dtype, like the reference's torch backend."""
    from benchmark_backends import PreparedCase, measure_cuda_device

    dtype = getattr(torch, INPUT_DTYPES[precision])
    m, n = a.shape[0], b.shape[1]
    with torch.cuda.stream(stream):
        left = torch.from_numpy(a).to(device=device, dtype=dtype)
        right = torch.from_numpy(b).to(device=device, dtype=dtype)
        out = torch.empty((m, n), dtype=torch.float32, device=device)
    half = precision in ("fp16", "bf16")

    def run():
        with torch.cuda.stream(stream):
            if half:
                torch.mm(left, right, out_dtype=torch.float32, out=out)
            else:
                torch.mm(left, right, out=out)
        return out

    def end_to_end():
        with torch.cuda.stream(stream):
            fa = torch.from_numpy(a).to(device).to(dtype)
            fb = torch.from_numpy(b).to(device).to(dtype)
            result = torch.mm(fa, fb, out_dtype=torch.float32) if half else torch.mm(fa, fb)
            return result.cpu().numpy()

    def output():
        stream.synchronize()
        return out.cpu().numpy()

    return PreparedCase(run, stream.synchronize, output, end_to_end, "cuda", {"library": "cublas"},
                        lambda w, r: measure_cuda_device(run, stream, w, r))


def main(argv=None) -> None:
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("--sizes", nargs="*", default=["1024"], help="M (square) or MxKxN")
    parser.add_argument("--precisions", nargs="+", default=list(PRECISIONS), choices=PRECISIONS)
    parser.add_argument("--backends", nargs="+", default=list(BACKENDS), choices=BACKENDS)
    parser.add_argument("--modes", nargs="+", default=list(MODES), choices=MODES)
    parser.add_argument("--seed", type=int, default=2026)
    parser.add_argument("--warmup", type=int, default=10)
    parser.add_argument("--repeats", type=int, default=21)
    parser.add_argument("--cpu-threads", type=int, default=0)
    parser.add_argument("--device", type=int, default=0)
    parser.add_argument("--library", default=None)
    parser.add_argument("--output", type=Path, default=Path("results"))
    args = parser.parse_args(argv)
    args.shapes = [parse_shape(s) for s in args.sizes]
    report = run(args)
    write_report(report, args.output)
    print(f"\nResults: {args.output.resolve()}")


if __name__ == "__main__":
    main()
