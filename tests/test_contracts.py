"""Host-side contracts of the backend (no GPU): the backend/precision table and
operand validation, restating tests/test_matmul.py:113-166 of the reference
for the checks that fire before any device work."""

from __future__ import annotations

import pytest
import torch

from precision import (BACKEND_PRECISIONS, CUDA_BACKENDS, INPUT_DTYPES, PRECISION_IDS, PRECISIONS,
                       unsupported_reason, validate_operands)


def test_precision_ids_match_the_reference_abi():
    assert PRECISION_IDS == {"fp32": 0, "tf32": 1, "fp16": 2, "bf16": 3}
    assert INPUT_DTYPES == {"fp32": "float32", "tf32": "float32", "fp16": "float16", "bf16": "bfloat16"}


def test_backend_precision_table():
    assert CUDA_BACKENDS == ("tcgen05", "ffma")
    assert BACKEND_PRECISIONS["tcgen05"] == ("tf32", "fp16", "bf16")
    assert BACKEND_PRECISIONS["ffma"] == ("fp32",)


@pytest.mark.parametrize("backend", CUDA_BACKENDS)
@pytest.mark.parametrize("precision", PRECISIONS)
def test_unsupported_reason(backend, precision):
    reason = unsupported_reason(backend, precision, (10, 0))
    assert (reason is None) == (precision in BACKEND_PRECISIONS[backend])
    if precision in BACKEND_PRECISIONS[backend]:
        assert "10.0" in unsupported_reason(backend, precision, (9, 0))
        assert "10.0" in unsupported_reason(backend, precision, (12, 0))
        assert unsupported_reason(backend, precision, None) is None
        assert unsupported_reason(backend, precision, (10, 0), target="cpu") is not None


def test_unknown_backend():
    assert unsupported_reason("wmma", "bf16", (10, 0)) is not None


def test_operand_contract_errors_before_device_checks():
    a = torch.ones((2, 3))
    b = torch.ones((3, 4))
    out = torch.empty((2, 4))
    cases = [
        (None, b, out, "fp32", TypeError),
        (a.flatten(), b, out, "fp32", ValueError),
        (a.double(), b, out, "fp32", TypeError),
        (a, b, out, "fp32", ValueError),                 # CPU tensors: wrong device
        (a.half(), b.half(), out, "fp16", ValueError),   # right dtypes, wrong device
        (a, b, out, "bf16", TypeError),                  # FP32 operands for BF16
        (a, b, out, "int8", ValueError),
    ]
    for index, (left, right, result, precision, error) in enumerate(cases):
        with pytest.raises(error):
            validate_operands(left, right, result, precision, 0)
