"""CPU oracle for the GEMM hot path (TEST INFRASTRUCTURE ONLY).

This module is the checker, never the thing measured or shipped.  Only the test
suite, ``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py`` may
import it.  The product path (``matrix-multiplication_b200``) never imports it and
has no CPU fallback.

It restates the reference's numerical contract from ``src/precision.py`` of
chudinovAI/matrix-multiplication:

* ``quantize_inputs``    -- ``src/precision.py:53-76``  (bit-exact RNE to TF32/BF16,
  numpy cast to FP16, optional TF32 ties-away, non-finite pass-through)
* ``reference_product``  -- ``src/precision.py:79-86``  (FP64 product of rounded inputs)
* ``GemmReference``      -- ``src/precision.py:99-161`` (gamma_K roundoff bound with
  u = FP32 epsilon, atol = rtol = 5e-4, TF32 candidate references, error report)

Parity pin: the restatement is checked against golden vectors produced by the
reference's own ``precision.py`` (``tests/golden/make_golden.py`` imports it and
writes ``tests/golden/precision_golden.npz``) and against the reference's own
known-answer tests (``tests/test_precision.py``), restated in
``tests/test_oracle.py``.

It also adds two helpers the reference does not have:

* ``baseline_bound_ratio`` -- the per-output bound ``c*K*u*sum|a||b|`` with u the
  unit roundoff of the *input* precision, measured against the unrounded FP32
  inputs (the bound stated for this backend's parity target);
* ``sampled_reference`` -- the same FP64 check restricted to a subset of output
  rows, so that 8192^3-class problems can be verified in seconds.
"""

from __future__ import annotations

import math

import numpy as np

PRECISIONS = ("fp32", "tf32", "fp16", "bf16")
RTOL = 5e-4
ATOL = 5e-4
# Unit roundoff of each input format (round to nearest): 2^-(p) with p the
# number of stored fraction bits + 1.
INPUT_UNIT_ROUNDOFF = {"fp32": 2.0**-24, "tf32": 2.0**-11, "fp16": 2.0**-11, "bf16": 2.0**-8}


def quantize_inputs(values, precision: str, *, tf32_ties: str = "even") -> np.ndarray:
    """FP32 representation of ``values`` rounded to ``precision`` (precision.py:53-76).

    TF32 keeps 10 fraction bits (drops 13), BF16 keeps 7 (drops 16).  Ties round
    to even by adding ``half-1 + lsb`` before truncation; ``tf32_ties="away"``
    adds exactly ``half``.  Infinities and NaNs (with payload) pass through.
    FP16 uses numpy's IEEE cast (RNE, subnormals kept, overflow to inf).
    """
    if precision not in PRECISIONS:
        raise ValueError(f"Unknown precision: {precision}")
    if tf32_ties not in ("even", "away") or (precision != "tf32" and tf32_ties != "even"):
        raise ValueError("TF32 tie policy must be even or away; other formats use even")
    x = np.asarray(values, dtype=np.float32)
    if precision == "fp32":
        return x
    if precision == "fp16":
        with np.errstate(over="ignore", invalid="ignore"):
            return x.astype(np.float16).astype(np.float32)
    dropped = 13 if precision == "tf32" else 16
    word = x.view(np.uint32).astype(np.uint64)
    half = np.uint64(1 << (dropped - 1))
    if tf32_ties == "away":
        increment = half
    else:
        increment = half - np.uint64(1) + ((word >> np.uint64(dropped)) & np.uint64(1))
    keep_mask = np.uint64(0xFFFFFFFF & ~((1 << dropped) - 1))
    rounded = ((word + increment) & keep_mask).astype(np.uint32)
    exponent_all_ones = (x.view(np.uint32) & np.uint32(0x7F800000)) == np.uint32(0x7F800000)
    out = np.where(exponent_all_ones, x.view(np.uint32), rounded)
    return out.astype(np.uint32, copy=False).view(np.float32)


def reference_product(a, b, precision: str, *, tf32_ties: str = "even") -> np.ndarray:
    """FP64 product of the rounded inputs (precision.py:79-86)."""
    left = quantize_inputs(a, precision, tf32_ties=tf32_ties)
    right = quantize_inputs(b, precision, tf32_ties=tf32_ties)
    if not np.isfinite(left).all() or not np.isfinite(right).all():
        raise ValueError(f"Input quantization to {precision} produced nonfinite values")
    return left.astype(np.float64) @ right.astype(np.float64)


def _relative_error(difference, reference):
    denominator = float(np.linalg.norm(reference))
    numerator = float(np.linalg.norm(difference))
    if denominator == 0:
        return 0.0 if numerator == 0 else None
    return numerator / denominator


def gamma(k: int, unit_roundoff: float) -> float:
    """gamma_k = k*u / (1 - k*u), or its exact form when k*u >= 1 (precision.py:125-130)."""
    ku = k * unit_roundoff
    return ku / (1 - ku) if ku < 1 else math.expm1(k * math.log1p(unit_roundoff))


class GemmReference:
    """FP64 input models and an FP32 accumulation-error bound (precision.py:99-131).

    ``verify`` follows precision.py:134-161: the allowance per output is
    ``ATOL + RTOL*|ref| + gamma_K(u=2^-23) * (|A| @ |B|)`` and the check fails when
    the largest ``|actual - ref| / allowance`` exceeds 1.
    """

    def __init__(self, a, b, precision: str, *, original=None):
        left = quantize_inputs(a, precision).astype(np.float64)
        right = quantize_inputs(b, precision).astype(np.float64)
        if not np.isfinite(left).all() or not np.isfinite(right).all():
            raise ValueError(f"Input quantization to {precision} produced nonfinite values")
        self.precision = precision
        self.original = original if original is not None else reference_product(a, b, "fp32")
        self.rounded = self.original if precision == "fp32" else left @ right
        self._references = {"rounded_inputs": self.rounded}
        magnitude_left, magnitude_right = np.abs(left), np.abs(right)
        if precision == "tf32":
            away_left = quantize_inputs(a, precision, tf32_ties="away").astype(np.float64)
            away_right = quantize_inputs(b, precision, tf32_ties="away").astype(np.float64)
            self._references["tf32_ties_away"] = away_left @ away_right
            self._references["original_fp32"] = self.original
            magnitude_left = np.maximum(np.maximum(magnitude_left, np.abs(away_left)), np.abs(a))
            magnitude_right = np.maximum(np.maximum(magnitude_right, np.abs(away_right)), np.abs(b))
        k = left.shape[1]
        unit_roundoff = float(np.finfo(np.float32).eps)
        self._roundoff_bound = gamma(k, unit_roundoff) * (magnitude_left @ magnitude_right)
        self._bound_max = float(self._roundoff_bound.max()) if self._roundoff_bound.size else 0.0

    @property
    def roundoff_bound(self) -> np.ndarray:
        return self._roundoff_bound

    def verify(self, actual, label: str, *, allow_tf32_library: bool = False) -> dict:
        """Check one FP32 output; raise RuntimeError when outside the allowance."""
        if (actual.shape != self.rounded.shape or actual.dtype != np.float32
                or not np.isfinite(actual).all()):
            raise RuntimeError(f"{label}: expected finite FP32 output of shape {self.rounded.shape}")
        result = actual.astype(np.float64)
        original_difference = result - self.original
        if allow_tf32_library and self.precision == "tf32":
            candidates = list(self._references.items())
        else:
            candidates = [("rounded_inputs", self.rounded)]
        best = None
        for name, reference in candidates:
            difference = result - reference
            allowance = ATOL + RTOL * np.abs(reference) + self._roundoff_bound
            scaled = float(np.max(np.abs(difference) / allowance))
            if best is None or scaled < best[0]:
                best = (scaled, name, reference, difference)
        scaled, name, reference, difference = best
        if scaled > 1:
            raise RuntimeError(f"{label}: incorrect GEMM (roundoff-aware tolerance ratio {scaled:.3g})")
        return {
            "max_abs_error": float(np.max(np.abs(original_difference))),
            "arithmetic_max_abs_error": float(np.max(np.abs(difference))),
            "max_tolerance_ratio": scaled,
            "arithmetic_reference": name,
            "roundoff_bound_max": self._bound_max,
            "relative_frobenius_error": _relative_error(original_difference, self.original),
            "arithmetic_relative_error": _relative_error(difference, reference),
            "quantization_relative_error": _relative_error(reference - self.original, self.original),
        }


def baseline_bound_ratio(a, b, actual, precision: str, *, c: float = 2.0) -> float:
    """Largest ``|actual - A@B| / (c*K*u_in*sum_k |a_ik||b_kj|)`` over all outputs.

    ``A@B`` is the FP64 product of the *unrounded* FP32 inputs and ``u_in`` the unit
    roundoff of the input precision, so the bound covers input rounding plus FP32
    accumulation.  A value <= 1 passes.  Outputs whose magnitude sum is zero must
    be exactly zero.
    """
    a64 = np.asarray(a, dtype=np.float32).astype(np.float64)
    b64 = np.asarray(b, dtype=np.float32).astype(np.float64)
    exact = a64 @ b64
    magnitude = np.abs(a64) @ np.abs(b64)
    k = a64.shape[1]
    bound = c * k * INPUT_UNIT_ROUNDOFF[precision] * magnitude
    error = np.abs(np.asarray(actual, dtype=np.float64) - exact)
    zero = bound == 0
    if np.any(error[zero] != 0):
        return float("inf")
    if not np.any(~zero):
        return 0.0
    return float(np.max(error[~zero] / bound[~zero]))


def sampled_reference(a, b, precision: str, rows) -> GemmReference:
    """``GemmReference`` of the output rows ``rows`` only (A[rows] @ B)."""
    rows = np.asarray(rows)
    return GemmReference(np.asarray(a)[rows], b, precision)


def seeded_uniform(shape, seed: int) -> np.ndarray:
    """U[-1,1) FP32 inputs from ``np.random.default_rng(seed)``."""
    return np.random.default_rng(seed).uniform(-1.0, 1.0, size=shape).astype(np.float32)


def seeded_normal(shape, seed: int, scale: float = 1.0) -> np.ndarray:
    """N(0, scale^2) FP32 inputs from ``np.random.default_rng(seed)``."""
    return (np.random.default_rng(seed).standard_normal(shape, dtype=np.float32) * np.float32(scale))
