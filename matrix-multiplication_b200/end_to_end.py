"""Host-to-host GEMM through the B200 library, with transfers overlapped.

The reference's end_to_end mode (src/benchmark_backends.py:295-307) copies the
FP32 host inputs to the device, converts them with ``torch .to(dtype)``, runs
the GEMM and copies C back, one step after the other.  ``HostMatmul`` produces
the same result with the PCIe link busy in both directions at once:

* B (FP32, pinned host) goes host->device first and is converted to the input
  format on the device (``matmul_convert``, round to nearest even);
* A follows in ``chunks`` row blocks on the same copy stream; each block is
  converted and multiplied (``matmul_launch``) on the compute stream as soon as
  it has arrived;
* each finished block of C goes device->host on a third stream while the next
  block of A is still arriving;
* the last row block can be split into ``tail_chunks`` smaller ones: what runs
  after the last byte of A has arrived is that block's conversion, GEMM and C
  copy, so a smaller last block shortens the step (8 blocks of 1024 rows at
  8192^3 BF16: the last C copy alone is 33.5 MB, ~0.65 ms on PCIe).

The call returns when C is in the caller's (pinned) host buffer.  Device
buffers are allocated once per instance and reused.
"""

from __future__ import annotations

import torch

from precision import BACKEND_PRECISIONS, INPUT_DTYPES
from sharded import chunk_rows


def row_blocks(m: int, chunks: int, tail_chunks: int = 1) -> list[tuple[int, int]]:
    """Contiguous, non-empty row blocks covering [0, m): ``chunks`` near-equal blocks
    with the last one split again into up to ``tail_chunks``."""
    ranges = chunk_rows(m, chunks)
    if tail_chunks > 1 and ranges:
        lo, hi = ranges.pop()
        ranges += [(lo + a, lo + b) for a, b in chunk_rows(hi - lo, tail_chunks)]
    return ranges


class HostMatmul:
    """C (host, FP32) = A (host, FP32) * B (host, FP32) computed in ``precision`` on one GPU."""

    def __init__(self, native, m: int, k: int, n: int, precision: str = "bf16", *, chunks: int = 4,
                 tail_chunks: int = 1, backend: str | None = None):
        self.native = native
        self.m, self.k, self.n = m, k, n
        self.precision = precision
        self.backend = backend or ("ffma" if precision == "fp32" else "tcgen05")
        if precision not in BACKEND_PRECISIONS[self.backend]:
            raise ValueError(f"{self.backend} does not support {precision}")
        self.device = torch.device("cuda", native.device)
        dtype = getattr(torch, INPUT_DTYPES[precision])
        self.ranges = row_blocks(m, chunks, tail_chunks)
        self.a32 = torch.empty((m, k), dtype=torch.float32, device=self.device)
        self.b32 = torch.empty((k, n), dtype=torch.float32, device=self.device)
        if precision == "fp32":
            self.a, self.b = self.a32, self.b32
        else:
            self.a = torch.empty((m, k), dtype=dtype, device=self.device)
            self.b = torch.empty((k, n), dtype=dtype, device=self.device)
        self.c = torch.empty((m, n), dtype=torch.float32, device=self.device)
        self.copy_in = torch.cuda.Stream(device=self.device)
        self.compute = torch.cuda.Stream(device=self.device)
        self.copy_out = torch.cuda.Stream(device=self.device)
        with torch.cuda.stream(self.compute):
            self.runs = [native.prepare(self.backend, self.a[lo:hi], self.b, self.c[lo:hi], precision=precision)
                         for lo, hi in self.ranges]

    @property
    def bytes_in(self) -> int:
        return 4 * (self.m * self.k + self.k * self.n)

    @property
    def bytes_out(self) -> int:
        return 4 * self.m * self.n

    def __call__(self, a_host: torch.Tensor, b_host: torch.Tensor, c_host: torch.Tensor) -> torch.Tensor:
        """Compute into ``c_host``; all three host tensors should be pinned FP32."""
        for name, t, shape in (("a", a_host, (self.m, self.k)), ("b", b_host, (self.k, self.n)),
                               ("c", c_host, (self.m, self.n))):
            if t.device.type != "cpu" or t.dtype != torch.float32 or tuple(t.shape) != shape:
                raise ValueError(f"{name}_host must be an FP32 CPU tensor of shape {shape}")
        convert = self.precision != "fp32"
        with torch.cuda.stream(self.copy_in):
            self.b32.copy_(b_host, non_blocking=True)
            b_ready = torch.cuda.Event()
            b_ready.record(self.copy_in)
            a_ready = []
            for lo, hi in self.ranges:
                self.a32[lo:hi].copy_(a_host[lo:hi], non_blocking=True)
                event = torch.cuda.Event()
                event.record(self.copy_in)
                a_ready.append(event)
        c_ready = []
        with torch.cuda.stream(self.compute):
            self.compute.wait_event(b_ready)
            if convert:
                self.native.convert(self.b32, self.b, self.precision)
            for (lo, hi), event, run in zip(self.ranges, a_ready, self.runs):
                self.compute.wait_event(event)
                if convert:
                    self.native.convert(self.a32[lo:hi], self.a[lo:hi], self.precision)
                run()
                done = torch.cuda.Event()
                done.record(self.compute)
                c_ready.append(done)
        with torch.cuda.stream(self.copy_out):
            for (lo, hi), event in zip(self.ranges, c_ready):
                self.copy_out.wait_event(event)
                c_host[lo:hi].copy_(self.c[lo:hi], non_blocking=True)
        self.copy_out.synchronize()
        return c_host
