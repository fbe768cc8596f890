"""The CPU oracle, pinned to the reference (no GPU needed).

* golden vectors written by the reference's own src/precision.py
  (tests/golden/make_golden.py);
* the reference's known-answer tests of tests/test_precision.py:12-102,
  restated against the oracle;
* the C restatement (oracle/gemm_oracle.c) cross-checked against the numpy one.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

import precision_oracle as po

FULL_SHAPES = ((1, 1, 1), (7, 13, 11), (35, 37, 67), (2, 2049, 3), (31, 33, 65))
SUMMARY_SHAPES = ((511, 257, 129), (513, 129, 577))


def _inputs(m, k, n):
    seed = 1000 * m + 10 * k + n
    a = np.random.default_rng(seed).uniform(-1, 1, (m, k)).astype(np.float32)
    b = np.random.default_rng(seed + 1).uniform(-1, 1, (k, n)).astype(np.float32)
    return a, b


# ------------------------------------------------------------------ golden vectors
@pytest.mark.parametrize("precision", po.PRECISIONS)
def test_quantize_matches_reference_bit_for_bit(golden, precision):
    with np.errstate(over="ignore", invalid="ignore"):
        got = po.quantize_inputs(golden["probe"], precision)
    np.testing.assert_array_equal(got.view(np.uint32), golden[f"quantize_{precision}"].view(np.uint32))


def test_tf32_ties_away_matches_reference(golden):
    got = po.quantize_inputs(golden["probe"], "tf32", tf32_ties="away")
    np.testing.assert_array_equal(got.view(np.uint32), golden["quantize_tf32_away"].view(np.uint32))


@pytest.mark.parametrize("shape", FULL_SHAPES)
@pytest.mark.parametrize("precision", po.PRECISIONS)
def test_gemm_reference_matches_reference(golden, shape, precision):
    tag = "x".join(map(str, shape))
    a, b = golden[f"a_{tag}"], golden[f"b_{tag}"]
    np.testing.assert_array_equal(a, _inputs(*shape)[0])
    reference = po.GemmReference(a, b, precision)
    np.testing.assert_array_equal(reference.rounded, golden[f"rounded_{tag}_{precision}"])
    np.testing.assert_allclose(reference.roundoff_bound, golden[f"bound_{tag}_{precision}"], rtol=1e-14, atol=0)
    report = reference.verify(reference.rounded.astype(np.float32), tag)
    assert report["max_tolerance_ratio"] == pytest.approx(float(golden[f"ratio_{tag}_{precision}"]), rel=1e-12)


@pytest.mark.parametrize("shape", SUMMARY_SHAPES)
@pytest.mark.parametrize("precision", po.PRECISIONS)
def test_ragged_checksums_match_reference(golden, shape, precision):
    tag = "x".join(map(str, shape))
    a, b = _inputs(*shape)
    reference = po.GemmReference(a, b, precision)
    rows = golden[f"sample_rows_{tag}"]
    np.testing.assert_allclose(reference.rounded[rows], golden[f"sample_{tag}_{precision}"], rtol=1e-13, atol=1e-13)
    checksum = np.array([reference.rounded.sum(), np.abs(reference.rounded).sum(),
                         reference.roundoff_bound.max(), reference.roundoff_bound.sum()])
    np.testing.assert_allclose(checksum, golden[f"checksum_{tag}_{precision}"], rtol=1e-12)


# ------------------------------------------------------------------ reference KATs
def test_tf32_and_bf16_signed_ties_round_to_even():
    for precision, fraction_bits in (("tf32", 10), ("bf16", 7)):
        step = 2.0 ** -fraction_bits
        source = np.array([1 + step / 2, 1 + 3 * step / 2, -1 - step / 2, -1 - 3 * step / 2], dtype=np.float32)
        expected = np.array([1, 1 + 2 * step, -1, -1 - 2 * step], dtype=np.float32)
        np.testing.assert_array_equal(po.quantize_inputs(source, precision), expected)


def test_signed_zero_and_nonfinite_values_are_not_reinterpreted():
    source = np.array([0.0, -0.0, np.inf, -np.inf, np.nan], dtype=np.float32)
    for precision in ("tf32", "fp16", "bf16"):
        rounded = po.quantize_inputs(source, precision)
        np.testing.assert_array_equal(rounded[:4].view(np.uint32), source[:4].view(np.uint32))
        assert np.isnan(rounded[4])


def test_fp16_subnormal_rounding_and_overflow():
    source = np.array([2.0**-24, 2.0**-25, -2.0**-25], dtype=np.float32)
    expected = np.array([2.0**-24, 0.0, -0.0], dtype=np.float32)
    np.testing.assert_array_equal(po.quantize_inputs(source, "fp16").view(np.uint32), expected.view(np.uint32))
    with pytest.raises(ValueError):
        po.GemmReference(np.array([[1e6]], dtype=np.float32), np.ones((1, 1), dtype=np.float32), "fp16")


def test_quantization_is_reported_separately_from_wrong_arithmetic():
    a = np.array([[1.003, -2.007], [0.125, 1.111]], dtype=np.float32)
    b = np.array([[0.333, 2.111], [-1.007, 0.125]], dtype=np.float32)
    reference = po.GemmReference(a, b, "bf16")
    correct = reference.rounded.astype(np.float32)
    metrics = reference.verify(correct, "bf16")
    assert metrics["quantization_relative_error"] > 0
    assert metrics["relative_frobenius_error"] > metrics["arithmetic_relative_error"]
    damaged = correct.copy()
    damaged[0, 0] += 0.1
    with pytest.raises(RuntimeError):
        reference.verify(damaged, "bf16")


def test_tf32_allows_ieee_only_when_the_backend_contract_permits_it():
    a = np.array([[1.0004, -1.0]], dtype=np.float32)
    b = np.array([[1.0004], [1.0]], dtype=np.float32)
    reference = po.GemmReference(a, b, "tf32")
    ieee_result = reference.original.astype(np.float32)
    with pytest.raises(RuntimeError):
        reference.verify(ieee_result, "forced TF32")
    metrics = reference.verify(ieee_result, "TF32 allowed", allow_tf32_library=True)
    assert metrics["arithmetic_reference"] == "original_fp32"
    assert metrics["quantization_relative_error"] == 0
    metrics = reference.verify(reference.rounded.astype(np.float32), "TF32 allowed", allow_tf32_library=True)
    assert metrics["arithmetic_reference"] == "rounded_inputs"
    with pytest.raises(RuntimeError):
        reference.verify(ieee_result + 0.1, "wrong TF32", allow_tf32_library=True)


def test_tf32_ties_away_is_a_distinct_strict_reference():
    values = np.array([1 + 2.0**-11, -1 - 2.0**-11], dtype=np.float32)
    away = po.quantize_inputs(values, "tf32", tf32_ties="away")
    np.testing.assert_array_equal(away, np.array([1 + 2.0**-10, -1 - 2.0**-10], dtype=np.float32))
    a = np.array([[values[0], -1.0]], dtype=np.float32)
    b = np.array([[4.0], [4.0]], dtype=np.float32)
    reference = po.GemmReference(a, b, "tf32")
    actual = np.array([[2.0**-8]], dtype=np.float32)
    with pytest.raises(RuntimeError):
        reference.verify(actual, "forced RNE")
    metrics = reference.verify(actual, "RNA", allow_tf32_library=True)
    assert metrics["arithmetic_reference"] == "tf32_ties_away"
    with pytest.raises(RuntimeError):
        reference.verify(actual + 0.1, "wrong RNA", allow_tf32_library=True)


def test_cancellation_respects_fp32_roundoff_but_rejects_wrong_results():
    a = np.array([[1e8, 1.0, -1e8]], dtype=np.float32)
    b = np.ones((3, 1), dtype=np.float32)
    reference = po.GemmReference(a, b, "fp32")
    actual = np.cumsum(a * b.T, axis=1, dtype=np.float32)[:, -1:]
    metrics = reference.verify(actual, "cancellation")
    assert metrics["max_abs_error"] == 1
    assert metrics["relative_frobenius_error"] == 1
    with pytest.raises(RuntimeError):
        reference.verify(np.array([[1000.0]], dtype=np.float32), "wrong cancellation")


def test_zero_reference_and_invalid_outputs():
    zero = np.zeros((2, 2), dtype=np.float32)
    reference = po.GemmReference(zero, np.ones((2, 2), dtype=np.float32), "fp32")
    assert reference.verify(zero, "zero")["relative_frobenius_error"] == 0
    assert reference.verify(np.full((2, 2), 1e-7, dtype=np.float32), "near zero")["relative_frobenius_error"] is None
    for invalid in (np.zeros((2, 3), dtype=np.float32), zero.astype(np.float64),
                    np.full((2, 2), np.nan, dtype=np.float32)):
        with pytest.raises(RuntimeError):
            reference.verify(invalid, "invalid")


# ------------------------------------------------------------------ a planted mistake
def test_oracle_rejects_a_planted_single_ulp_class_error():
    """A wrong product in one output of a large-K case must fail the oracle."""
    a, b = _inputs(31, 33, 65)
    reference = po.GemmReference(a, b, "bf16")
    good = reference.rounded.astype(np.float32)
    reference.verify(good, "good")
    bad = good.copy()
    bad[30, 64] += 0.05
    with pytest.raises(RuntimeError):
        reference.verify(bad, "planted")


# ------------------------------------------------------------------ baseline bound
@pytest.mark.parametrize("precision", po.PRECISIONS)
def test_baseline_bound_accepts_rounded_products_and_rejects_garbage(precision):
    a, b = _inputs(35, 37, 67)
    reference = po.GemmReference(a, b, precision)
    ratio = po.baseline_bound_ratio(a, b, reference.rounded.astype(np.float32), precision, c=2.0)
    assert ratio <= 1.0
    # The bound is c*K*u_in*sum|a||b| (loose for BF16 at K=37, about 0.29*sum|a||b|):
    # an error of K*sum|a||b| must fail it for every format.
    magnitude = np.abs(a.astype(np.float64)) @ np.abs(b.astype(np.float64))
    bad = (reference.rounded + 37 * magnitude).astype(np.float32)
    assert po.baseline_bound_ratio(a, b, bad, precision, c=2.0) > 1.0


# ------------------------------------------------------------------ C restatement
def _f32p(array):
    return array.ctypes.data_as(ctypes.POINTER(ctypes.c_float))


@pytest.mark.parametrize("precision", po.PRECISIONS)
def test_c_oracle_quantize_agrees_with_numpy_oracle(oracle_c, golden, precision):
    probe = np.ascontiguousarray(golden["probe"], dtype=np.float32)
    out = np.empty_like(probe)
    oracle_c.oracle_quantize(_f32p(probe), _f32p(out), probe.size, po.PRECISIONS.index(precision), 0)
    np.testing.assert_array_equal(out.view(np.uint32), golden[f"quantize_{precision}"].view(np.uint32))


def test_c_oracle_quantize_ties_away(oracle_c, golden):
    probe = np.ascontiguousarray(golden["probe"], dtype=np.float32)
    out = np.empty_like(probe)
    oracle_c.oracle_quantize(_f32p(probe), _f32p(out), probe.size, 1, 1)
    np.testing.assert_array_equal(out.view(np.uint32), golden["quantize_tf32_away"].view(np.uint32))


def test_c_oracle_gemm_and_verify_agree_with_numpy_oracle(oracle_c):
    a, b = _inputs(35, 37, 67)
    qa = np.ascontiguousarray(po.quantize_inputs(a, "bf16"))
    qb = np.ascontiguousarray(po.quantize_inputs(b, "bf16"))
    rows = np.arange(35, dtype=np.int64)
    out = np.empty((35, 67), dtype=np.float64)
    oracle_c.oracle_gemm_rows(_f32p(qa), _f32p(qb), out.ctypes.data_as(ctypes.POINTER(ctypes.c_double)),
                              rows.ctypes.data_as(ctypes.POINTER(ctypes.c_int64)), 35, 37, 67)
    reference = po.GemmReference(a, b, "bf16")
    np.testing.assert_allclose(out, reference.rounded, rtol=1e-14, atol=1e-14)
    actual = reference.rounded.astype(np.float32)
    ratio = oracle_c.oracle_verify_rows(_f32p(qa), _f32p(qb), _f32p(actual),
                                        rows.ctypes.data_as(ctypes.POINTER(ctypes.c_int64)), 35, 37, 67)
    assert ratio == pytest.approx(reference.verify(actual, "c")["max_tolerance_ratio"], rel=1e-9)
