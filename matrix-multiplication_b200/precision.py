"""Precision and operand contracts of the B200 GEMM backend.

Host-side mirror of the contract half of the reference's ``src/precision.py``
(the numerical oracle half lives in ``oracle/`` and is test-only):

* ``PRECISIONS`` / ``INPUT_DTYPES`` / ``PRECISION_IDS``  -- precision.py:8-10
* ``BACKEND_PRECISIONS`` / ``unsupported_reason``       -- precision.py:16-50
* ``validate_operands``                                 -- precision.py:164-194
* ``torch_precision``                                   -- precision.py:217-234

The backends registered here are this library's: ``tcgen05`` (TF32, FP16, BF16
on fifth-generation tensor cores) and ``ffma`` (pedantic FP32).  Both need a
compute capability 10.0 device (B200, sm_100a).
"""

from __future__ import annotations

from contextlib import contextmanager

PRECISIONS = ("fp32", "tf32", "fp16", "bf16")
INPUT_DTYPES = {"fp32": "float32", "tf32": "float32", "fp16": "float16", "bf16": "bfloat16"}
PRECISION_IDS = {name: index for index, name in enumerate(PRECISIONS)}
CUDA_BACKENDS = ("tcgen05", "ffma")
BACKEND_PRECISIONS = {
    "tcgen05": ("tf32", "fp16", "bf16"),
    "ffma": ("fp32",),
}
REQUIRED_CAPABILITY = (10, 0)
RTOL = 5e-4
ATOL = 5e-4
_INT_MAX = 2**31 - 1


def unsupported_reason(backend: str, precision: str, capability: tuple[int, int] | None,
                       *, target: str = "cuda") -> str | None:
    """Why ``backend`` cannot run ``precision`` here, or None (precision.py:30-50)."""
    if backend not in BACKEND_PRECISIONS:
        return f"unknown backend: {backend}"
    if target != "cuda":
        return f"{backend} is a CUDA backend"
    if precision not in BACKEND_PRECISIONS[backend]:
        return f"{backend} supports {', '.join(BACKEND_PRECISIONS[backend])}, not {precision}"
    if capability is not None and tuple(capability) != REQUIRED_CAPABILITY:
        return (f"{backend} requires NVIDIA compute capability "
                f"{REQUIRED_CAPABILITY[0]}.{REQUIRED_CAPABILITY[1]} (B200, sm_100a)")
    return None


def validate_operands(a, b, out, precision: str, device: int) -> tuple[int, int, int]:
    """Validate the row-major CUDA tensor contract once (precision.py:164-194).

    Raises TypeError for a wrong type or dtype and ValueError for a wrong rank,
    device, layout, shape, size or an output that overlaps an input.
    """
    import torch

    if precision not in PRECISIONS:
        raise ValueError(f"Unknown precision: {precision}")
    input_dtype = getattr(torch, INPUT_DTYPES[precision])
    for name, tensor, dtype in (("a", a, input_dtype), ("b", b, input_dtype), ("out", out, torch.float32)):
        if not isinstance(tensor, torch.Tensor):
            raise TypeError(f"{name} must be a torch.Tensor")
        if tensor.ndim != 2:
            raise ValueError(f"{name} must be a two-dimensional matrix")
        if tensor.dtype != dtype:
            raise TypeError(f"{name} must have dtype {dtype}")
        if tensor.device.type != "cuda" or tensor.device.index != device:
            raise ValueError(f"{name} must be on cuda:{device}")
        if not tensor.is_contiguous():
            raise ValueError(f"{name} must be contiguous")
    m, k = a.shape
    k2, n = b.shape
    if k != k2 or tuple(out.shape) != (m, n):
        raise ValueError("expected a=(m, k), b=(k, n), and out=(m, n)")
    if any(size <= 0 or size > _INT_MAX for size in (m, k, n)):
        raise ValueError("matrix dimensions must be positive and fit in a C int")
    begin = out.data_ptr()
    end = begin + out.numel() * out.element_size()
    for name, tensor in (("a", a), ("b", b)):
        address = tensor.data_ptr()
        if begin < address + tensor.numel() * tensor.element_size() and address < end:
            raise ValueError(f"out must not overlap {name}")
    return m, k, n


@contextmanager
def torch_precision(torch, precision: str):
    """Set torch's FP32/TF32 and reduction policy for one case, then restore it."""
    if precision not in PRECISIONS:
        raise ValueError(f"Unknown precision: {precision}")
    backend = torch.backends.cuda.matmul
    previous = backend.fp32_precision
    fp16_reduction = backend.allow_fp16_reduced_precision_reduction
    bf16_reduction = backend.allow_bf16_reduced_precision_reduction
    try:
        backend.fp32_precision = "tf32" if precision == "tf32" else "ieee"
        backend.allow_fp16_reduced_precision_reduction = False
        backend.allow_bf16_reduced_precision_reduction = False
        yield
    finally:
        backend.fp32_precision = previous
        backend.allow_fp16_reduced_precision_reduction = fp16_reduction
        backend.allow_bf16_reduced_precision_reduction = bf16_reduction
