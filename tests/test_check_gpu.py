"""The GPU FP64 checker (matmul_check_fp64), pinned to the CPU oracle, and the
full-output verification it makes possible at benchmark sizes (needs a B200).

The checker restates the reference's GemmReference.verify on the GPU.  It is
trusted only because it agrees with the CPU oracle on every shape and precision
below, including outputs with a planted error; the CPU oracle stays the ground
truth.  With it, every output of the 8192^3 and LLM-shaped problems is checked,
not only sampled rows.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import precision_oracle as po
from precision import BACKEND_PRECISIONS, INPUT_DTYPES

pytestmark = pytest.mark.gpu

PLANS = [(backend, precision) for backend in ("tcgen05", "ffma") for precision in BACKEND_PRECISIONS[backend]]


def _device_operands(a_np, b_np, precision):
    dtype = getattr(torch, INPUT_DTYPES[precision])
    return (torch.from_numpy(a_np).to(device="cuda", dtype=dtype),
            torch.from_numpy(b_np).to(device="cuda", dtype=dtype))


@pytest.mark.parametrize("backend,precision", PLANS)
@pytest.mark.parametrize("shape", ((1, 1, 1), (31, 33, 65), (129, 65, 257), (300, 1000, 520), (513, 129, 577)))
def test_gpu_checker_agrees_with_cpu_oracle(native, backend, precision, shape):
    m, k, n = shape
    a_np = po.seeded_uniform((m, k), 7 * m + k)
    b_np = po.seeded_uniform((k, n), 5 * n + k)
    a, b = _device_operands(a_np, b_np, precision)
    out = torch.empty((m, n), dtype=torch.float32, device="cuda")
    native.prepare(backend, a, b, out, precision=precision)()
    torch.cuda.synchronize()
    report = po.GemmReference(a_np, b_np, precision).verify(out.cpu().numpy(), "cpu oracle")
    ratio, max_err = native.check_fp64(a, b, out, precision)
    assert ratio == pytest.approx(report["max_tolerance_ratio"], rel=1e-6, abs=1e-12)
    assert max_err == pytest.approx(report["arithmetic_max_abs_error"], rel=1e-6, abs=1e-12)
    assert ratio <= 1.0


@pytest.mark.parametrize("precision", ("tf32", "bf16", "fp32"))
def test_gpu_checker_flags_a_planted_error_like_the_oracle(native, precision):
    m, k, n = 200, 300, 400
    a_np = po.seeded_uniform((m, k), 3)
    b_np = po.seeded_uniform((k, n), 4)
    a, b = _device_operands(a_np, b_np, precision)
    out = torch.empty((m, n), dtype=torch.float32, device="cuda")
    native.prepare("ffma" if precision == "fp32" else "tcgen05", a, b, out, precision=precision)()
    torch.cuda.synchronize()
    out[123, 321] += 0.05
    ratio, _ = native.check_fp64(a, b, out, precision)
    assert ratio > 1.0
    with pytest.raises(RuntimeError):
        po.GemmReference(a_np, b_np, precision).verify(out.cpu().numpy(), "planted")
    out[17, 5] = float("nan")
    assert native.check_fp64(a, b, out, precision)[0] == float("inf")


@pytest.mark.parametrize("backend,precision,shape", [
    ("tcgen05", "bf16", (8192, 8192, 8192)),
    ("tcgen05", "fp16", (8192, 8192, 8192)),
    ("tcgen05", "tf32", (4096, 4096, 4096)),
    ("ffma", "fp32", (4096, 4096, 4096)),
    ("tcgen05", "bf16", (8192, 8192, 28672)),
    ("tcgen05", "fp16", (4096, 14336, 4096)),
    ("tcgen05", "bf16", (16, 8192, 8192)),
    ("tcgen05", "fp16", (16, 8192, 8192)),
])
def test_every_output_at_benchmark_sizes(native, backend, precision, shape):
    """Full verification of every output (the benchmark's N(0, 1/sqrt(K)) inputs)."""
    m, k, n = shape
    gen = torch.Generator(device="cuda")
    gen.manual_seed(m + k + n)
    dtype = getattr(torch, INPUT_DTYPES[precision])
    a32 = torch.randn((m, k), generator=gen, device="cuda") * k ** -0.5
    b32 = torch.randn((k, n), generator=gen, device="cuda") * k ** -0.5
    a = torch.empty((m, k), dtype=dtype, device="cuda")
    b = torch.empty((k, n), dtype=dtype, device="cuda")
    native.convert(a32, a, precision)
    native.convert(b32, b, precision)
    del a32, b32
    out = torch.full((m, n), float("nan"), dtype=torch.float32, device="cuda")
    native.prepare(backend, a, b, out, precision=precision)()
    ratio, max_err = native.check_fp64(a, b, out, precision)
    assert np.isfinite(ratio) and ratio <= 1.0, (ratio, max_err)
