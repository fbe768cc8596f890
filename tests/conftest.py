"""Shared test setup: import paths, the `gpu` marker and library fixtures.

Tests marked ``gpu`` need a B200 and call the library through its C-ABI; the
rest run on any machine (oracle, host logic, library loading and exports).
"""

from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
PACKAGE = ROOT / "matrix-multiplication_b200"
ORACLE = ROOT / "oracle"
for path in (PACKAGE, ORACLE, ROOT):
    if str(path) not in sys.path:
        sys.path.insert(0, str(path))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device with compute capability 10.0 (B200)")


@pytest.fixture(scope="session")
def library_path() -> Path:
    """The built library; built here when missing or stale (nvcc cross-compiles)."""
    import build as native_build

    return native_build.build()


@pytest.fixture(scope="session")
def oracle_c():
    """The C restatement of the oracle (oracle/_lib/liboracle.so), built on demand."""
    import ctypes
    import subprocess

    lib = ORACLE / "_lib" / "liboracle.so"
    if not lib.exists() or lib.stat().st_mtime < (ORACLE / "gemm_oracle.c").stat().st_mtime:
        subprocess.run(["make", "-s", "-C", str(ORACLE), "oracle"], check=True)
    handle = ctypes.CDLL(str(lib))
    f32p = ctypes.POINTER(ctypes.c_float)
    f64p = ctypes.POINTER(ctypes.c_double)
    i64p = ctypes.POINTER(ctypes.c_int64)
    handle.oracle_quantize.argtypes = [f32p, f32p, ctypes.c_size_t, ctypes.c_int, ctypes.c_int]
    handle.oracle_quantize.restype = None
    handle.oracle_gemm_rows.argtypes = [f32p, f32p, f64p, i64p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64]
    handle.oracle_gemm_rows.restype = None
    handle.oracle_verify_rows.argtypes = [f32p, f32p, f32p, i64p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64]
    handle.oracle_verify_rows.restype = ctypes.c_double
    return handle


@pytest.fixture(scope="session")
def golden():
    import numpy as np

    with np.load(ROOT / "tests" / "golden" / "precision_golden.npz") as data:
        return {key: data[key] for key in data.files}


def _gpu_ready() -> bool:
    try:
        import torch
    except ImportError:
        return False
    return torch.cuda.is_available() and torch.cuda.get_device_capability(0) == (10, 0)


@pytest.fixture(scope="session")
def gpu_ready():
    if not _gpu_ready():
        pytest.fail("GPU tests need a compute capability 10.0 device; run with -m 'not gpu' elsewhere")
    return True


@pytest.fixture()
def native(gpu_ready, library_path):
    from gpumat import NativeMatmul

    context = NativeMatmul(library_path)
    yield context
    status = context.device_status() if not context.closed else 0
    context.close()
    assert status == 0, f"a kernel reported a bounded-wait timeout (status {status:#x})"
