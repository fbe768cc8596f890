"""Prepared GEMM cases and the CUDA-graph device timer for the B200 backends.

Mirror of the CUDA parts of the reference's ``src/benchmark_backends.py``:

* ``DEVICE_BATCH`` and ``measure_cuda_device`` -- benchmark_backends.py:17,49-69:
  one CUDA graph holds external start/end events around ``DEVICE_BATCH`` calls;
  each sample is the event interval divided by the batch.
* ``PreparedCase`` / ``cuda_case`` -- benchmark_backends.py:72-88,279-310: the
  host FP32 inputs are placed on the device in the input dtype, a resident FP32
  output is allocated, and ``end_to_end`` runs the whole host-to-host path.

The end-to-end path differs in one respect: inputs go host->device as FP32
(pinned) and are converted on the device by the library's ``matmul_convert``
(round to nearest even), instead of torch's ``.to(dtype)``.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Callable

import torch

from precision import INPUT_DTYPES

DEVICE_BATCH = 10


def measure_cuda_device(call, stream, warmup: int, repeats: int) -> list[float]:
    """Milliseconds per call from CUDA events around a captured batch of calls."""
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
    samples = []
    for _ in range(repeats):
        graph.replay()
        end.synchronize()
        samples.append(start.elapsed_time(end) / DEVICE_BATCH)
    del graph
    return samples


@dataclass
class PreparedCase:
    run: Callable
    synchronize: Callable
    output: Callable
    end_to_end: Callable
    execution_device: str
    config: dict | None = None
    device_samples: Callable | None = None


def cuda_case(native, backend: str, precision: str, a, b, stream) -> PreparedCase:
    """Resident device case plus an end_to_end closure for host FP32 ``a``, ``b``."""
    device = torch.device("cuda", native.device)
    dtype = getattr(torch, INPUT_DTYPES[precision])
    m, n = a.shape[0], b.shape[1]
    with torch.cuda.stream(stream):
        left = torch.from_numpy(a).to(device=device, dtype=dtype)
        right = torch.from_numpy(b).to(device=device, dtype=dtype)
        out = torch.empty((m, n), dtype=torch.float32, device=device)
        run = native.prepare(backend, left, right, out, precision=precision)
    config = native.configuration(backend, precision)
    pinned_a = torch.from_numpy(a).pin_memory()
    pinned_b = torch.from_numpy(b).pin_memory()

    def end_to_end():
        with torch.cuda.stream(stream):
            fa = pinned_a.to(device, non_blocking=True)
            fb = pinned_b.to(device, non_blocking=True)
            ta = torch.empty(fa.shape, dtype=dtype, device=device)
            tb = torch.empty(fb.shape, dtype=dtype, device=device)
            native.convert(fa, ta, precision)
            native.convert(fb, tb, precision)
            result = torch.empty((m, n), dtype=torch.float32, device=device)
            native.prepare(backend, ta, tb, result, precision=precision)()
            host = result.cpu()
        return host.numpy()

    def timer(warmup, repeats):
        return measure_cuda_device(run, stream, warmup, repeats)

    def output():
        stream.synchronize()
        return out.cpu().numpy()

    return PreparedCase(run, stream.synchronize, output, end_to_end, "cuda", config, timer)
