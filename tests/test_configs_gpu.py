"""Parity on the benchmark configurations exactly as stated (needs a B200).

Every single-GPU configuration of the benchmark, at its stated size, input
distribution and precision, through the C-ABI, against the FP64 oracle
(``GemmReference.verify``, the reference's src/precision.py:99-161) and the
backend's own bound |C - A.B| <= c.K.u_in.sum|a||b| (c = 2):

* FP32 1024^3, A and B i.i.d. U[-1,1) drawn in that order from
  ``np.random.default_rng(0)``, on the FFMA kernel;
* the ragged partial-tile shapes 31x33x65, 511x257x129, 513x129x577 in FP32 and
  BF16 (U[-1,1) FP32 from a seed, rounded to BF16 for the BF16 case);
* the square sweep 64..4096 (powers of two) at FP32, TF32, FP16 and BF16,
  U[-1,1) from a seed, rounded to the input precision;
* 8192^3, 16x8192x8192, 8192x8192x28672 and 4096x14336x4096 in BF16 and FP16,
  inputs N(0, 1/sqrt(K)) from a seed.

Outputs up to 1024^3 are checked in full on the CPU.  Above that every output
is checked by ``matmul_check_fp64`` (the GPU form of the same FP64 check, itself
pinned to the CPU oracle by test_check_gpu.py) and sampled rows by the CPU
oracle as well.  The reference checks every implementation and precision on its
fixed shapes the same way (tests/test_matmul.py:28-51).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import precision_oracle as po
from precision import INPUT_DTYPES

pytestmark = pytest.mark.gpu

BASELINE_C = 2.0
SQUARE_SIZES = (64, 128, 256, 512, 1024, 2048, 4096)
SWEEP_PRECISIONS = ("fp32", "tf32", "fp16", "bf16")
LLM_SHAPES = ((8192, 8192, 8192), (16, 8192, 8192), (8192, 8192, 28672), (4096, 14336, 4096))
RAGGED_SHAPES = ((31, 33, 65), (511, 257, 129), (513, 129, 577))
CPU_FULL_LIMIT = 1024 ** 3        # m*k*n checked in full on the CPU


def _backend(precision):
    return "ffma" if precision == "fp32" else "tcgen05"


def _device_inputs(a32: torch.Tensor, b32: torch.Tensor, precision: str, native):
    """FP32 device inputs -> the input dtype of ``precision`` (round to nearest even)."""
    dtype = getattr(torch, INPUT_DTYPES[precision])
    a = torch.empty(a32.shape, dtype=dtype, device="cuda")
    b = torch.empty(b32.shape, dtype=dtype, device="cuda")
    native.convert(a32, a, precision)
    native.convert(b32, b, precision)
    return a, b


def _run(native, precision, a, b):
    m, n = a.shape[0], b.shape[1]
    out = torch.full((m, n), float("nan"), dtype=torch.float32, device="cuda")
    native.prepare(_backend(precision), a, b, out, precision=precision)()
    torch.cuda.synchronize()
    return out


def _check(native, precision, a_np, b_np, a, b, out, label):
    """Full CPU check up to CPU_FULL_LIMIT; above it the GPU FP64 check of every
    output plus a CPU check of sampled rows."""
    m, k = a_np.shape
    n = b_np.shape[1]
    if m * k * n <= CPU_FULL_LIMIT:
        actual = out.cpu().numpy()
        po.GemmReference(a_np, b_np, precision).verify(actual, label)
        assert po.baseline_bound_ratio(a_np, b_np, actual, precision, c=BASELINE_C) <= 1.0
        return
    assert torch.isfinite(out).all().item(), f"{label}: non-finite output"
    ratio, max_err = native.check_fp64(a, b, out, precision)
    assert ratio <= 1.0, f"{label}: GPU FP64 check ratio {ratio} (max |err| {max_err})"
    rows = np.unique(np.concatenate([[0, m - 1], np.random.default_rng(m * 3 + n).integers(0, m, 6)]))
    sampled = out[torch.from_numpy(rows).cuda()].cpu().numpy()
    po.sampled_reference(a_np, b_np, precision, rows).verify(sampled, f"{label} sampled rows")
    assert po.baseline_bound_ratio(a_np[rows], b_np, sampled, precision, c=BASELINE_C) <= 1.0


def test_config_fp32_1024_seed0(native):
    """FP32 1024^3, U[-1,1) from default_rng(0) (A first, then B), on the numpy-comparable path."""
    rng = np.random.default_rng(0)
    a_np = rng.uniform(-1.0, 1.0, (1024, 1024)).astype(np.float32)
    b_np = rng.uniform(-1.0, 1.0, (1024, 1024)).astype(np.float32)
    a = torch.from_numpy(a_np).cuda()
    b = torch.from_numpy(b_np).cuda()
    out = _run(native, "fp32", a, b)
    _check(native, "fp32", a_np, b_np, a, b, out, "config fp32 1024^3 seed 0")


@pytest.mark.parametrize("precision", ("fp32", "bf16"))
@pytest.mark.parametrize("shape", RAGGED_SHAPES)
def test_config_ragged(native, shape, precision):
    m, k, n = shape
    a_np = po.seeded_uniform((m, k), 10 * m + k)
    b_np = po.seeded_uniform((k, n), 10 * n + k + 1)
    a, b = _device_inputs(torch.from_numpy(a_np).cuda(), torch.from_numpy(b_np).cuda(), precision, native)
    out = _run(native, precision, a, b)
    _check(native, precision, a_np, b_np, a, b, out, f"ragged {m}x{k}x{n} {precision}")


@pytest.mark.parametrize("precision", SWEEP_PRECISIONS)
@pytest.mark.parametrize("size", SQUARE_SIZES)
def test_config_square_sweep(native, size, precision):
    a_np = po.seeded_uniform((size, size), 2 * size)
    b_np = po.seeded_uniform((size, size), 2 * size + 1)
    a, b = _device_inputs(torch.from_numpy(a_np).cuda(), torch.from_numpy(b_np).cuda(), precision, native)
    out = _run(native, precision, a, b)
    _check(native, precision, a_np, b_np, a, b, out, f"square {size}^3 {precision}")


@pytest.mark.parametrize("precision", ("bf16", "fp16"))
@pytest.mark.parametrize("shape", LLM_SHAPES)
def test_config_large_and_llm_shapes(native, shape, precision):
    m, k, n = shape
    a_np = po.seeded_normal((m, k), 3 * m + k, scale=k ** -0.5)
    b_np = po.seeded_normal((k, n), 3 * n + k + 1, scale=k ** -0.5)
    a, b = _device_inputs(torch.from_numpy(a_np).cuda(), torch.from_numpy(b_np).cuda(), precision, native)
    out = _run(native, precision, a, b)
    _check(native, precision, a_np, b_np, a, b, out, f"{m}x{k}x{n} {precision} N(0,1/sqrt(K))")
