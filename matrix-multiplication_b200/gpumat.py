"""ctypes loader for the B200 GEMM library (``build/b200_matmul.so``).

Mirror of the reference's ``src/gpumat.py`` (``NativeMatmul``, :15-155) with
the same constructor, ``configuration()``, ``prepare()``, ``close()`` and
error behaviour:

* the library path defaults to ``<repo>/build/b200_matmul.so`` and a missing
  file raises FileNotFoundError (there is no fallback of any kind);
* the ABI version must be 3 (gpumat.py:31-44);
* ``prepare`` validates the operands (TypeError / ValueError), captures the
  current stream, calls ``record_stream`` on every tensor and returns a
  ``run()`` closure that keeps a, b and out alive and raises RuntimeError
  on a nonzero native return or after ``close()`` (gpumat.py:119-155).

Implementation names map to this library's ids: ``tcgen05`` -> 7, ``ffma`` -> 8.
"""

from __future__ import annotations

import ctypes
import json
from pathlib import Path

import torch

from precision import PRECISION_IDS, unsupported_reason, validate_operands

_IMPLEMENTATIONS = {"tcgen05": 7, "ffma": 8}
_ERROR_SIZE = 1024
_INT_MAX = 2**31 - 1
DEFAULT_LIBRARY = Path(__file__).resolve().parent.parent / "build" / "b200_matmul.so"


class NativeMatmul:
    """Own a native B200 matmul context for one CUDA device."""

    def __init__(self, library: str | Path | None = None, device: int = 0):
        if isinstance(device, bool) or not isinstance(device, int) or not 0 <= device <= _INT_MAX:
            raise ValueError("device must be a non-negative CUDA device index")
        path = Path(library) if library is not None else DEFAULT_LIBRARY
        if not path.is_file():
            raise FileNotFoundError(
                f"Native matmul library not found at {path}. Run "
                "`python matrix-multiplication_b200/build.py` or pass a library path."
            )
        try:
            self._library = ctypes.CDLL(str(path.resolve()))
        except OSError as exc:
            raise OSError(f"Could not load native matmul library at {path}: {exc}") from exc
        try:
            abi_version = self._library.matmul_abi_version
        except AttributeError as exc:
            raise RuntimeError(f"Native matmul library at {path} has no ABI version; rebuild it.") from exc
        abi_version.argtypes = []
        abi_version.restype = ctypes.c_int
        version = abi_version()
        if version != 3:
            raise RuntimeError(f"Native matmul library at {path} has ABI version {version}, expected 3; rebuild it.")
        self.path = path.resolve()
        _bind(self._library)
        self._device = device
        self._context = None
        error = ctypes.create_string_buffer(_ERROR_SIZE)
        context = self._library.matmul_create(device, error, len(error))
        if not context:
            raise RuntimeError(self._error_message("matmul_create", error))
        self._context = context
        self._capability = torch.cuda.get_device_capability(device)

    @staticmethod
    def _error_message(operation, error):
        detail = error.value.decode("utf-8", errors="replace")
        return f"{operation} failed: {detail or 'unknown native error'}"

    @property
    def device(self) -> int:
        return self._device

    def close(self):
        """Destroy the context once; prepared operations cannot be used afterward."""
        context = self._context
        if context is not None:
            self._context = None
            error = ctypes.create_string_buffer(_ERROR_SIZE)
            if self._library.matmul_destroy(context, error, len(error)) != 0:
                raise RuntimeError(self._error_message("matmul_destroy", error))

    def __enter__(self):
        if self._context is None:
            raise RuntimeError("NativeMatmul context is closed")
        return self

    def __exit__(self, exc_type, exc_value, traceback):
        self.close()

    def __del__(self):
        try:
            if getattr(self, "_context", None) is not None:
                self.close()
        except Exception:
            pass

    def configuration(self, implementation: str, precision: str = "fp32") -> dict:
        """Return the native kernel's launch geometry and staging policy."""
        if self._context is None:
            raise RuntimeError("NativeMatmul context is closed")
        if not isinstance(implementation, str) or implementation not in _IMPLEMENTATIONS:
            raise ValueError(f"unknown implementation: {implementation!r}")
        if not isinstance(precision, str) or precision not in PRECISION_IDS:
            raise ValueError(f"unknown precision: {precision!r}")
        reason = unsupported_reason(implementation, precision, self._capability)
        if reason is not None:
            raise ValueError(reason)
        return kernel_info(self._library, implementation, precision)

    def prepare(self, implementation: str, a: torch.Tensor, b: torch.Tensor, out: torch.Tensor,
                *, precision: str = "fp32"):
        """Prepare an asynchronous operation on the current CUDA stream."""
        if self._context is None:
            raise RuntimeError("NativeMatmul context is closed")
        if not isinstance(implementation, str) or implementation not in _IMPLEMENTATIONS:
            raise ValueError(f"unknown implementation: {implementation!r}")
        m, k, n = validate_operands(a, b, out, precision, self._device)
        reason = unsupported_reason(implementation, precision, self._capability)
        if reason is not None:
            raise ValueError(reason)
        a_ptr = ctypes.c_void_p(a.data_ptr())
        b_ptr = ctypes.c_void_p(b.data_ptr())
        out_ptr = ctypes.c_void_p(out.data_ptr())
        stream = torch.cuda.current_stream(self._device)
        stream_ptr = ctypes.c_void_p(stream.cuda_stream)
        for tensor in (a, b, out):
            tensor.record_stream(stream)
        implementation_id = _IMPLEMENTATIONS[implementation]
        precision_id = PRECISION_IDS[precision]
        launch = self._library.matmul_launch
        error = ctypes.create_string_buffer(_ERROR_SIZE)

        def run():
            _ = a, b, stream
            context = self._context
            if context is None:
                raise RuntimeError("NativeMatmul context is closed")
            if launch(context, implementation_id, precision_id, a_ptr, b_ptr, out_ptr, m, k, n,
                      stream_ptr, error, len(error)) != 0:
                raise RuntimeError(self._error_message("matmul_launch", error))
            return out

        return run

    def plan(self, implementation: str, m: int, k: int, n: int, precision: str = "fp32") -> dict:
        """The launch ``prepare(...)()`` would make for an m x k x n problem (kernel,
        tile, K splits; the FFMA plan assumes 16-byte aligned operands)."""
        if self._context is None:
            raise RuntimeError("NativeMatmul context is closed")
        if not isinstance(implementation, str) or implementation not in _IMPLEMENTATIONS:
            raise ValueError(f"unknown implementation: {implementation!r}")
        if not isinstance(precision, str) or precision not in PRECISION_IDS:
            raise ValueError(f"unknown precision: {precision!r}")
        result = ctypes.create_string_buffer(_ERROR_SIZE)
        error = ctypes.create_string_buffer(_ERROR_SIZE)
        if self._library.matmul_plan(self._context, _IMPLEMENTATIONS[implementation], PRECISION_IDS[precision],
                                     m, k, n, result, len(result), error, len(error)) != 0:
            raise RuntimeError(self._error_message("matmul_plan", error))
        return json.loads(result.value)

    def set_sm_limit(self, sms: int) -> None:
        """Run later tensor-core launches on at most ``sms`` SMs (0 = all of them)."""
        if self._context is None:
            raise RuntimeError("NativeMatmul context is closed")
        if isinstance(sms, bool) or not isinstance(sms, int):
            raise TypeError("sms must be an int")
        error = ctypes.create_string_buffer(_ERROR_SIZE)
        if self._library.matmul_set_sm_limit(self._context, sms, error, len(error)) != 0:
            raise RuntimeError(self._error_message("matmul_set_sm_limit", error))

    def convert(self, src: torch.Tensor, dst: torch.Tensor, precision: str) -> torch.Tensor:
        """Convert FP32 ``src`` into ``dst`` (the input dtype of ``precision``) on the device.

        BF16/FP16 round to nearest even; TF32 keeps FP32 storage rounded to 10
        fraction bits (ties to even); FP32 copies.
        """
        if self._context is None:
            raise RuntimeError("NativeMatmul context is closed")
        if precision not in PRECISION_IDS:
            raise ValueError(f"Unknown precision: {precision}")
        from precision import INPUT_DTYPES

        if src.dtype != torch.float32 or dst.dtype != getattr(torch, INPUT_DTYPES[precision]):
            raise TypeError("src must be float32 and dst the input dtype of the precision")
        for tensor in (src, dst):
            if tensor.device.type != "cuda" or tensor.device.index != self._device or not tensor.is_contiguous():
                raise ValueError(f"tensors must be contiguous on cuda:{self._device}")
        if src.numel() != dst.numel():
            raise ValueError("src and dst must have the same number of elements")
        stream = torch.cuda.current_stream(self._device)
        error = ctypes.create_string_buffer(_ERROR_SIZE)
        if self._library.matmul_convert(self._context, PRECISION_IDS[precision], ctypes.c_void_p(src.data_ptr()),
                                        ctypes.c_void_p(dst.data_ptr()), src.numel(),
                                        ctypes.c_void_p(stream.cuda_stream), error, len(error)) != 0:
            raise RuntimeError(self._error_message("matmul_convert", error))
        return dst

    def check_fp64(self, a: torch.Tensor, b: torch.Tensor, out: torch.Tensor, precision: str) -> tuple[float, float]:
        """Verify ``out`` against an FP64 product of the rounded inputs on the GPU.

        Returns (largest tolerance ratio, largest absolute error); a ratio <= 1
        passes the reference's roundoff-aware allowance.  Synchronizes.
        """
        if self._context is None:
            raise RuntimeError("NativeMatmul context is closed")
        m, k, n = validate_operands(a, b, out, precision, self._device)
        stream = torch.cuda.current_stream(self._device)
        result = (ctypes.c_double * 2)()
        error = ctypes.create_string_buffer(_ERROR_SIZE)
        if self._library.matmul_check_fp64(self._context, PRECISION_IDS[precision], ctypes.c_void_p(a.data_ptr()),
                                           ctypes.c_void_p(b.data_ptr()), ctypes.c_void_p(out.data_ptr()), m, k, n,
                                           ctypes.c_void_p(stream.cuda_stream), result, error, len(error)) != 0:
            raise RuntimeError(self._error_message("matmul_check_fp64", error))
        return float(result[0]), float(result[1])

    def device_status(self, clear: bool = True) -> int:
        """Synchronize and return the device status word (0 = no kernel timed out)."""
        if self._context is None:
            raise RuntimeError("NativeMatmul context is closed")
        status = ctypes.c_uint(0)
        error = ctypes.create_string_buffer(_ERROR_SIZE)
        if self._library.matmul_device_status(self._context, int(bool(clear)), ctypes.byref(status),
                                              error, len(error)) != 0:
            raise RuntimeError(self._error_message("matmul_device_status", error))
        return int(status.value)


def _bind(library) -> None:
    library.matmul_create.argtypes = [ctypes.c_int, ctypes.c_char_p, ctypes.c_size_t]
    library.matmul_create.restype = ctypes.c_void_p
    library.matmul_destroy.argtypes = [ctypes.c_void_p, ctypes.c_char_p, ctypes.c_size_t]
    library.matmul_destroy.restype = ctypes.c_int
    library.matmul_launch.argtypes = [
        ctypes.c_void_p, ctypes.c_int, ctypes.c_int,
        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
        ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p,
        ctypes.c_char_p, ctypes.c_size_t,
    ]
    library.matmul_launch.restype = ctypes.c_int
    library.matmul_kernel_info.argtypes = [
        ctypes.c_int, ctypes.c_int, ctypes.c_char_p, ctypes.c_size_t, ctypes.c_char_p, ctypes.c_size_t,
    ]
    library.matmul_kernel_info.restype = ctypes.c_int
    library.matmul_convert.argtypes = [
        ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p,
        ctypes.c_char_p, ctypes.c_size_t,
    ]
    library.matmul_convert.restype = ctypes.c_int
    library.matmul_device_status.argtypes = [
        ctypes.c_void_p, ctypes.c_int, ctypes.POINTER(ctypes.c_uint), ctypes.c_char_p, ctypes.c_size_t,
    ]
    library.matmul_device_status.restype = ctypes.c_int
    library.matmul_check_fp64.argtypes = [
        ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int,
        ctypes.c_int, ctypes.c_void_p, ctypes.POINTER(ctypes.c_double), ctypes.c_char_p, ctypes.c_size_t,
    ]
    library.matmul_check_fp64.restype = ctypes.c_int
    library.matmul_plan.argtypes = [
        ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
        ctypes.c_char_p, ctypes.c_size_t, ctypes.c_char_p, ctypes.c_size_t,
    ]
    library.matmul_plan.restype = ctypes.c_int
    library.matmul_set_sm_limit.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_char_p, ctypes.c_size_t]
    library.matmul_set_sm_limit.restype = ctypes.c_int


def kernel_info(library, implementation: str, precision: str) -> dict:
    """``matmul_kernel_info`` as a dict (needs no GPU)."""
    result = ctypes.create_string_buffer(_ERROR_SIZE)
    error = ctypes.create_string_buffer(_ERROR_SIZE)
    if library.matmul_kernel_info(_IMPLEMENTATIONS[implementation], PRECISION_IDS[precision], result, len(result),
                                  error, len(error)) != 0:
        raise RuntimeError(NativeMatmul._error_message("matmul_kernel_info", error))
    return json.loads(result.value)


def load_library(library: str | Path | None = None):
    """Load and bind the library without creating a device context."""
    path = Path(library) if library is not None else DEFAULT_LIBRARY
    if not path.is_file():
        raise FileNotFoundError(f"Native matmul library not found at {path}")
    handle = ctypes.CDLL(str(path.resolve()))
    _bind(handle)
    return handle
