"""The C-ABI library without a GPU: it loads, exports every declared symbol,
reports ABI 3 and kernel geometry, and rejects bad calls with the reference's
error convention (src/matmul.cu:36-47, :213-272)."""

from __future__ import annotations

import ctypes
import json
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "b200_matmul.h"


def declared_functions() -> list[str]:
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:int\s+|void\s*\*\s*)(\w+)\s*\(", text, flags=re.M)))


@pytest.fixture(scope="module")
def lib(library_path):
    from gpumat import load_library

    return load_library(library_path)


def test_header_declares_the_reference_exports():
    names = declared_functions()
    for name in ("matmul_abi_version", "matmul_kernel_info", "matmul_create", "matmul_destroy", "matmul_launch"):
        assert name in names


def test_library_exports_every_declared_symbol(lib):
    for name in declared_functions():
        assert hasattr(lib, name), name


def test_abi_version_is_three(lib):
    lib.matmul_abi_version.restype = ctypes.c_int
    assert lib.matmul_abi_version() == 3


def _info(lib, implementation, precision, size=1024):
    out = ctypes.create_string_buffer(size)
    err = ctypes.create_string_buffer(256)
    rc = lib.matmul_kernel_info(implementation, precision, out, len(out), err, len(err))
    return rc, out.value.decode(), err.value.decode()


@pytest.mark.parametrize("implementation,precision", [(7, 1), (7, 2), (7, 3), (8, 0)])
def test_kernel_info_reports_reference_keys(lib, implementation, precision):
    rc, text, err = _info(lib, implementation, precision)
    assert rc == 0 and err == ""
    info = json.loads(text)
    for key in ("implementation", "precision", "tile_m", "tile_n", "tile_k", "threads", "warp_tile_m",
                "warp_tile_n", "microtile_m", "microtile_n", "buffering", "load_method", "tensor_cores"):
        assert key in info
    assert info["tensor_cores"] is (implementation == 7)
    assert info["precision"] == ("fp32", "tf32", "fp16", "bf16")[precision]


@pytest.mark.parametrize("implementation,precision", [(7, 0), (8, 1), (8, 3), (2, 0), (6, 3), (9, 0), (7, 4), (-1, 0)])
def test_kernel_info_rejects_unsupported_combinations(lib, implementation, precision):
    rc, text, err = _info(lib, implementation, precision)
    assert rc == 1 and text == ""
    assert err.startswith("matmul_kernel_info: ")


def test_kernel_info_reports_a_small_buffer(lib):
    rc, text, err = _info(lib, 7, 3, size=16)
    assert rc == 1 and text == ""
    assert "too small" in err


def test_null_context_is_rejected(lib):
    err = ctypes.create_string_buffer(256)
    rc = lib.matmul_launch(None, 7, 3, None, None, None, 1, 1, 1, None, err, len(err))
    assert rc == 1 and err.value.decode() == "matmul_launch: context is null"
    rc = lib.matmul_destroy(None, err, len(err))
    assert rc == 1 and err.value.decode() == "matmul_destroy: context is null"
    rc = lib.matmul_convert(None, 3, None, None, 1, None, err, len(err))
    assert rc == 1
    status = ctypes.c_uint(0)
    rc = lib.matmul_device_status(None, 0, ctypes.byref(status), err, len(err))
    assert rc == 1


def test_error_buffer_may_be_null(lib):
    assert lib.matmul_launch(None, 7, 3, None, None, None, 1, 1, 1, None, None, 0) == 1


def test_create_fails_cleanly_without_a_usable_device(lib):
    import torch

    if torch.cuda.is_available():
        pytest.skip("a CUDA device is present")
    err = ctypes.create_string_buffer(256)
    assert not lib.matmul_create(0, err, len(err))
    assert err.value.decode().startswith("cudaSetDevice: ")


def test_loader_refuses_a_missing_library(tmp_path):
    from gpumat import NativeMatmul

    with pytest.raises(FileNotFoundError):
        NativeMatmul(tmp_path / "missing.so")


def test_loader_rejects_bad_device_index(library_path):
    from gpumat import NativeMatmul

    for device in (-1, True, 1.0, "0"):
        with pytest.raises(ValueError):
            NativeMatmul(library_path, device=device)


def test_library_is_sm100a_only():
    import build

    cmd = build.command()
    assert "arch=compute_100a,code=sm_100a" in cmd
