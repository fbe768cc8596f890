"""ctypes binding of the B200 GEMM library (``build/b200_matmul.so``).

The reference's harness reaches its CUDA library through ``src/gpumat.py``
(``NativeMatmul``, :15-155).  This module offers the same public surface, so
that harness code written against it runs unchanged:

    NativeMatmul(library=None, device=0)
        .configuration(implementation, precision)   -> dict (kernel geometry)
        .prepare(implementation, a, b, out, *, precision) -> run()
        .close(), ``with NativeMatmul(...) as native:``

and it fails the same way: FileNotFoundError for a missing library,
RuntimeError for a wrong ABI version, ValueError / TypeError for bad arguments
and operand contracts (``precision.validate_operands``), and
``RuntimeError("<operation> failed: <detail>")`` for a nonzero native return or
a closed context.

The structure is this library's own:

* ``EXPORTS`` declares every C entry point of ``include/b200_matmul.h`` once,
  with its argument and result types; ``Library`` loads one copy of the .so per
  path, checks the ABI version and binds the whole table.
* Every export except ``matmul_abi_version`` and ``matmul_create`` returns 0/1
  and takes a caller-owned error buffer as its last two arguments;
  ``Library.invoke`` supplies the buffer and turns a nonzero return into the
  RuntimeError above.
* ``NativeMatmul`` owns one device context.  ``prepare`` returns a
  ``PreparedLaunch``: the launch's arguments marshalled once (pointers, sizes,
  the current stream, an error buffer), plus references to the tensors and the
  stream, so that a call costs one ctypes call and the operands stay alive as
  long as the launch does.

Implementation names map to this library's ids: ``tcgen05`` -> 7, ``ffma`` -> 8.
There is no fallback of any kind: without the library nothing runs.
"""

from __future__ import annotations

import ctypes
import json
import threading
from pathlib import Path

import torch

from precision import INPUT_DTYPES, PRECISION_IDS, unsupported_reason, validate_operands

ABI_VERSION = 3
IMPLEMENTATION_IDS = {"tcgen05": 7, "ffma": 8}
DEFAULT_LIBRARY = Path(__file__).resolve().parent.parent / "build" / "b200_matmul.so"
ERROR_BYTES = 1024
JSON_BYTES = 1024
_INT_MAX = 2**31 - 1

_P = ctypes.c_void_p
_I = ctypes.c_int
_ERROR_ARGS = (ctypes.c_char_p, ctypes.c_size_t)
_MATRIX_CALL = (_P, _I, _I, _P, _P, _P, _I, _I, _I, _P)

# name -> (argument types without the trailing error buffer, result type, takes an error buffer)
EXPORTS: dict[str, tuple[tuple, object, bool]] = {
    "matmul_abi_version": ((), ctypes.c_int, False),
    "matmul_kernel_info": ((_I, _I, ctypes.c_char_p, ctypes.c_size_t), ctypes.c_int, True),
    "matmul_create": ((_I,), _P, True),
    "matmul_destroy": ((_P,), ctypes.c_int, True),
    "matmul_launch": (_MATRIX_CALL, ctypes.c_int, True),
    "matmul_launch_noalloc": (_MATRIX_CALL, ctypes.c_int, True),
    "matmul_convert": ((_P, _I, _P, _P, ctypes.c_size_t, _P), ctypes.c_int, True),
    "matmul_device_status": ((_P, _I, ctypes.POINTER(ctypes.c_uint)), ctypes.c_int, True),
    "matmul_check_fp64": ((_P, _I, _P, _P, _P, _I, _I, _I, _P, ctypes.POINTER(ctypes.c_double)), ctypes.c_int,
                          True),
    "matmul_plan": ((_P, _I, _I, _I, _I, _I, ctypes.c_char_p, ctypes.c_size_t), ctypes.c_int, True),
    "matmul_set_sm_limit": ((_P, _I), ctypes.c_int, True),
    "matmul_set_wait_limit": ((_P, ctypes.c_ulonglong), ctypes.c_int, True),
    "matmul_peer_push": ((_P, _P, ctypes.POINTER(_P), _I, ctypes.c_size_t, _I, _P), ctypes.c_int, True),
}


def _library_path(library: str | Path | None) -> Path:
    path = Path(library) if library is not None else DEFAULT_LIBRARY
    if not path.is_file():
        raise FileNotFoundError(
            f"Native matmul library not found at {path}. Build it with "
            "`python matrix-multiplication_b200/build.py` or pass a library path.")
    return path.resolve()


class Library:
    """One loaded copy of the library with every export of ``EXPORTS`` bound."""

    _open: dict[Path, "Library"] = {}
    _lock = threading.Lock()

    def __init__(self, path: Path):
        try:
            self.cdll = ctypes.CDLL(str(path))
        except OSError as exc:
            raise OSError(f"Could not load native matmul library at {path}: {exc}") from exc
        self.path = path
        missing = [name for name in EXPORTS if not hasattr(self.cdll, name)]
        if "matmul_abi_version" in missing:
            raise RuntimeError(f"Native matmul library at {path} has no ABI version; rebuild it.")
        self.cdll.matmul_abi_version.argtypes = []
        self.cdll.matmul_abi_version.restype = ctypes.c_int
        version = self.cdll.matmul_abi_version()
        if version != ABI_VERSION:
            raise RuntimeError(f"Native matmul library at {path} has ABI version {version}, expected "
                               f"{ABI_VERSION}; rebuild it.")
        if missing:
            raise RuntimeError(f"Native matmul library at {path} lacks {', '.join(missing)}; rebuild it.")
        for name, (argtypes, restype, with_error) in EXPORTS.items():
            function = getattr(self.cdll, name)
            function.argtypes = list(argtypes) + (list(_ERROR_ARGS) if with_error else [])
            function.restype = restype

    @classmethod
    def open(cls, library: str | Path | None = None) -> "Library":
        path = _library_path(library)
        with cls._lock:
            if path not in cls._open:
                cls._open[path] = cls(path)
            return cls._open[path]

    @staticmethod
    def failure(operation: str, error) -> RuntimeError:
        detail = error.value.decode("utf-8", errors="replace")
        return RuntimeError(f"{operation} failed: {detail or 'unknown native error'}")

    def invoke(self, name: str, *args):
        """Call export ``name`` with a fresh error buffer; RuntimeError on a nonzero return."""
        error = ctypes.create_string_buffer(ERROR_BYTES)
        result = getattr(self.cdll, name)(*args, error, len(error))
        if name == "matmul_create":
            if not result:
                raise self.failure(name, error)
        elif result != 0:
            raise self.failure(name, error)
        return result

    def kernel_info(self, implementation: str, precision: str) -> dict:
        """``matmul_kernel_info`` as a dict (needs no GPU)."""
        text = ctypes.create_string_buffer(JSON_BYTES)
        self.invoke("matmul_kernel_info", IMPLEMENTATION_IDS[implementation], PRECISION_IDS[precision], text,
                    len(text))
        return json.loads(text.value)


class PreparedLaunch:
    """One GEMM launch with its arguments marshalled once (``NativeMatmul.prepare``).

    Calling it enqueues ``matmul_launch`` on the stream that was current at
    ``prepare`` time and returns ``out``.  It holds a, b, out and the stream, so
    none of them can be freed while the launch object exists.
    """

    __slots__ = ("_owner", "_function", "_arguments", "_error", "_tensors", "_stream", "out")

    def __init__(self, owner: "NativeMatmul", implementation: int, precision: int, a, b, out, m, k, n, stream):
        self._owner = owner
        self._function = owner.library.matmul_launch
        self._error = ctypes.create_string_buffer(ERROR_BYTES)
        self._arguments = (implementation, precision, _P(a.data_ptr()), _P(b.data_ptr()), _P(out.data_ptr()),
                           m, k, n, _P(stream.cuda_stream), self._error, len(self._error))
        self._tensors = (a, b, out)
        self._stream = stream
        self.out = out

    def __call__(self):
        handle = self._owner._handle
        if handle is None:
            raise RuntimeError("NativeMatmul context is closed")
        if self._function(handle, *self._arguments) != 0:
            raise Library.failure("matmul_launch", self._error)
        return self.out


class NativeMatmul:
    """A context of the native B200 GEMM library on one CUDA device."""

    def __init__(self, library: str | Path | None = None, device: int = 0):
        if isinstance(device, bool) or not isinstance(device, int) or not 0 <= device <= _INT_MAX:
            raise ValueError("device must be a non-negative CUDA device index")
        self._handle = None
        self._lib = Library.open(library)
        self.path = self._lib.path
        self._device = device
        self._handle = _P(self._lib.invoke("matmul_create", device))
        self._capability = torch.cuda.get_device_capability(device)

    # ---------------------------------------------------------------- lifetime
    @property
    def device(self) -> int:
        return self._device

    @property
    def library(self):
        """The bound ctypes library (every export of ``EXPORTS``)."""
        return self._lib.cdll

    @property
    def handle(self):
        """The native context pointer; RuntimeError once the context is closed."""
        if self._handle is None:
            raise RuntimeError("NativeMatmul context is closed")
        return self._handle

    @property
    def closed(self) -> bool:
        return self._handle is None

    def close(self) -> None:
        """Destroy the context (once); prepared launches fail afterwards."""
        handle, self._handle = self._handle, None
        if handle is not None:
            self._lib.invoke("matmul_destroy", handle)

    def __enter__(self):
        self.handle
        return self

    def __exit__(self, *exc_info):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ---------------------------------------------------------------- argument checks
    def _implementation_id(self, implementation) -> int:
        if not isinstance(implementation, str) or implementation not in IMPLEMENTATION_IDS:
            raise ValueError(f"unknown implementation: {implementation!r}")
        return IMPLEMENTATION_IDS[implementation]

    def _require_supported(self, implementation: str, precision: str) -> None:
        reason = unsupported_reason(implementation, precision, self._capability)
        if reason is not None:
            raise ValueError(reason)

    # ---------------------------------------------------------------- the reference's surface
    def configuration(self, implementation: str, precision: str = "fp32") -> dict:
        """The kernel's geometry and staging policy (``matmul_kernel_info``)."""
        self.handle
        self._implementation_id(implementation)
        if not isinstance(precision, str) or precision not in PRECISION_IDS:
            raise ValueError(f"unknown precision: {precision!r}")
        self._require_supported(implementation, precision)
        return self._lib.kernel_info(implementation, precision)

    def prepare(self, implementation: str, a: torch.Tensor, b: torch.Tensor, out: torch.Tensor, *,
                precision: str = "fp32") -> PreparedLaunch:
        """Validate the operands once and return a launch on the current CUDA stream."""
        self.handle
        implementation_id = self._implementation_id(implementation)
        m, k, n = validate_operands(a, b, out, precision, self._device)
        self._require_supported(implementation, precision)
        stream = torch.cuda.current_stream(self._device)
        for tensor in (a, b, out):
            tensor.record_stream(stream)
        return PreparedLaunch(self, implementation_id, PRECISION_IDS[precision], a, b, out, m, k, n, stream)

    # ---------------------------------------------------------------- this library's additions
    def plan(self, implementation: str, m: int, k: int, n: int, precision: str = "fp32") -> dict:
        """The launch ``prepare(...)()`` would make for an m x k x n problem (kernel,
        tile, K splits; the FFMA plan assumes 16-byte aligned operands)."""
        handle = self.handle
        implementation_id = self._implementation_id(implementation)
        if not isinstance(precision, str) or precision not in PRECISION_IDS:
            raise ValueError(f"unknown precision: {precision!r}")
        text = ctypes.create_string_buffer(JSON_BYTES)
        self._lib.invoke("matmul_plan", handle, implementation_id, PRECISION_IDS[precision], m, k, n, text,
                         len(text))
        return json.loads(text.value)

    def set_sm_limit(self, sms: int) -> None:
        """Run later tensor-core launches on at most ``sms`` SMs (0 = all of them)."""
        handle = self.handle
        if isinstance(sms, bool) or not isinstance(sms, int):
            raise TypeError("sms must be an int")
        self._lib.invoke("matmul_set_sm_limit", handle, sms)

    def set_wait_limit(self, nanoseconds: int) -> None:
        """Limit the tensor-core kernels' progress waits (0 = the default 2 s)."""
        handle = self.handle
        if isinstance(nanoseconds, bool) or not isinstance(nanoseconds, int) or nanoseconds < 0:
            raise ValueError("the wait limit is a non-negative number of nanoseconds")
        self._lib.invoke("matmul_set_wait_limit", handle, nanoseconds)

    def convert(self, src: torch.Tensor, dst: torch.Tensor, precision: str) -> torch.Tensor:
        """Convert FP32 ``src`` into ``dst`` (the input dtype of ``precision``) on the device.

        BF16/FP16 round to nearest even; TF32 keeps FP32 storage rounded to 10
        fraction bits (ties to even); FP32 copies.
        """
        handle = self.handle
        if precision not in PRECISION_IDS:
            raise ValueError(f"Unknown precision: {precision}")
        if src.dtype != torch.float32 or dst.dtype != getattr(torch, INPUT_DTYPES[precision]):
            raise TypeError("src must be float32 and dst the input dtype of the precision")
        for tensor in (src, dst):
            if tensor.device.type != "cuda" or tensor.device.index != self._device or not tensor.is_contiguous():
                raise ValueError(f"tensors must be contiguous on cuda:{self._device}")
        if src.numel() != dst.numel():
            raise ValueError("src and dst must have the same number of elements")
        stream = torch.cuda.current_stream(self._device)
        self._lib.invoke("matmul_convert", handle, PRECISION_IDS[precision], _P(src.data_ptr()),
                         _P(dst.data_ptr()), src.numel(), _P(stream.cuda_stream))
        return dst

    def check_fp64(self, a: torch.Tensor, b: torch.Tensor, out: torch.Tensor, precision: str) -> tuple[float, float]:
        """Verify ``out`` against an FP64 product of the rounded inputs on the GPU.

        Returns (largest tolerance ratio, largest absolute error); a ratio <= 1
        passes the reference's roundoff-aware allowance.  Synchronizes.
        """
        handle = self.handle
        m, k, n = validate_operands(a, b, out, precision, self._device)
        stream = torch.cuda.current_stream(self._device)
        result = (ctypes.c_double * 2)()
        self._lib.invoke("matmul_check_fp64", handle, PRECISION_IDS[precision], _P(a.data_ptr()),
                         _P(b.data_ptr()), _P(out.data_ptr()), m, k, n, _P(stream.cuda_stream), result)
        return float(result[0]), float(result[1])

    def peer_push(self, src_ptr: int, peer_ptrs: list[int], nbytes: int, stream=None, ctas: int = 0) -> None:
        """Copy ``nbytes`` at device address ``src_ptr`` into each address of
        ``peer_ptrs`` (peers' mapped buffers) on ``stream`` (default: current)."""
        handle = self.handle
        stream = stream if stream is not None else torch.cuda.current_stream(self._device)
        dsts = (_P * max(1, len(peer_ptrs)))(*[_P(p) for p in peer_ptrs])
        self._lib.invoke("matmul_peer_push", handle, _P(src_ptr), dsts, len(peer_ptrs), nbytes, ctas,
                         _P(stream.cuda_stream))

    def device_status(self, clear: bool = True) -> int:
        """Synchronize and return the device status word (0 = no kernel's wait ran out)."""
        handle = self.handle
        status = ctypes.c_uint(0)
        self._lib.invoke("matmul_device_status", handle, int(bool(clear)), ctypes.byref(status))
        return int(status.value)


def kernel_info(library, implementation: str, precision: str) -> dict:
    """``matmul_kernel_info`` of a library loaded with ``load_library`` (needs no GPU)."""
    text = ctypes.create_string_buffer(JSON_BYTES)
    error = ctypes.create_string_buffer(ERROR_BYTES)
    if library.matmul_kernel_info(IMPLEMENTATION_IDS[implementation], PRECISION_IDS[precision], text, len(text),
                                  error, len(error)) != 0:
        raise Library.failure("matmul_kernel_info", error)
    return json.loads(text.value)


def load_library(library: str | Path | None = None):
    """The bound ctypes library, without creating a device context."""
    return Library.open(library).cdll
