"""The allocation-free entry point, matmul_launch_noalloc (needs a B200).

Some callers cannot allocate device memory at call time: their framework has
already reserved nearly all of it in its own pool, and one more allocation
would fail or force the pool to give memory back.  For them the library has a second launch
entry point whose scratch (repacked copies of unaligned operands) lives in
a fixed 32 MiB array compiled into the library.  These tests call it through
the C-ABI and check that, on two calls in a row, it gives the same output as
matmul_launch (within the tolerance used by every other parity test here, and
against the FP64 oracle) on every kind of scratch use: repacked unaligned TF32,
FP16 and BF16 operands for the single-CTA, split-K and skinny kernels; and that a
problem too large for the array is rejected with a clear error.  The file name makes pytest collect it last.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

import precision_oracle as po
from precision import INPUT_DTYPES, PRECISION_IDS

pytestmark = pytest.mark.gpu

TCGEN05 = 7
RTOL = ATOL = 5e-4


def _bind(lib):
    lib.matmul_launch_noalloc.argtypes = [
        ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
        ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_char_p, ctypes.c_size_t]
    lib.matmul_launch_noalloc.restype = ctypes.c_int


def _operands(precision, m, k, n, offset):
    a_np = po.seeded_uniform((m, k), 500 + m)
    b_np = po.seeded_uniform((k, n), 600 + n)
    dtype = getattr(torch, INPUT_DTYPES[precision])
    if offset:
        a = torch.empty(m * k + 1, dtype=dtype, device="cuda")[1:].view(m, k)
        b = torch.empty(k * n + 1, dtype=dtype, device="cuda")[1:].view(k, n)
    else:
        a = torch.empty((m, k), dtype=dtype, device="cuda")
        b = torch.empty((k, n), dtype=dtype, device="cuda")
    a.copy_(torch.from_numpy(a_np))
    b.copy_(torch.from_numpy(b_np))
    return a_np, b_np, a, b


def _launch(fn, native, precision, a, b, out):
    err = ctypes.create_string_buffer(1024)
    m, k = a.shape
    n = b.shape[1]
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = fn(native.handle, TCGEN05, PRECISION_IDS[precision], ctypes.c_void_p(a.data_ptr()),
            ctypes.c_void_p(b.data_ptr()), ctypes.c_void_p(out.data_ptr()), m, k, n, stream, err, len(err))
    return rc, err.value.decode()


# Only operands TMA cannot address (base not 16-byte aligned, or a row pitch that
# is not a multiple of 16 bytes) are copied into scratch; TF32 problems up to
# m*k*n = 2^25 run on the FFMA kernel and need none, so every TF32 case here is
# larger than that and has an unaligned operand.
@pytest.mark.parametrize("precision,shape,offset", [
    ("tf32", (384, 260, 517), False),     # scratch: repacked B (n % 4 != 0; single-CTA tiles)
    ("tf32", (257, 300, 515), True),      # scratch: repacked A and B (offset bases)
    ("tf32", (512, 1026, 512), False),    # scratch: repacked A (k % 4 != 0), 2 MiB
    ("tf32", (48, 1024, 1022), False),    # scratch: repacked B feeding the skinny (m <= 64) kernel
    ("bf16", (513, 129, 577), True),      # scratch: repacked unaligned operands
    ("bf16", (130, 4099, 258), True),     # scratch: repacked operands of a split-K launch
    ("fp16", (256, 512, 512), False),     # aligned: no scratch needed
])
def test_noalloc_matches_matmul_launch_on_two_calls(native, precision, shape, offset):
    lib = native.library
    _bind(lib)
    m, k, n = shape
    plan = native.plan("tcgen05", m, k, n, precision=precision)
    assert plan["kernel"] in ("tc_single", "tc2_pair", "tc_skinny"), plan
    a_np, b_np, a, b = _operands(precision, m, k, n, offset)
    expected = torch.full((m, n), float("nan"), dtype=torch.float32, device="cuda")
    rc, msg = _launch(lib.matmul_launch, native, precision, a, b, expected)
    assert rc == 0, msg
    reference = po.GemmReference(a_np, b_np, precision)
    for call in range(2):
        out = torch.full((m, n), float("nan"), dtype=torch.float32, device="cuda")
        rc, msg = _launch(lib.matmul_launch_noalloc, native, precision, a, b, out)
        assert rc == 0, msg
        torch.cuda.synchronize()
        got = out.cpu().numpy()
        np.testing.assert_allclose(got, expected.cpu().numpy(), rtol=RTOL, atol=ATOL)
        reference.verify(got, f"noalloc {precision} call {call}")


def test_noalloc_rejects_problems_beyond_the_fixed_array(native):
    lib = native.library
    _bind(lib)
    m, k, n = 4096, 4096, 4097            # repacked TF32 B (n % 4 != 0) needs 64 MiB > 32 MiB
    a = torch.zeros((m, k), dtype=torch.float32, device="cuda")
    b = torch.zeros((k, n), dtype=torch.float32, device="cuda")
    out = torch.zeros((m, n), dtype=torch.float32, device="cuda")
    rc, msg = _launch(lib.matmul_launch_noalloc, native, "tf32", a, b, out)
    assert rc == 1
    assert msg.startswith("matmul_launch_noalloc: this problem needs")
    assert "fixed" in msg


def test_noalloc_accepts_only_the_tcgen05_implementation(native):
    lib = native.library
    _bind(lib)
    a = torch.ones((2, 2), dtype=torch.float32, device="cuda")
    out = torch.empty((2, 2), dtype=torch.float32, device="cuda")
    err = ctypes.create_string_buffer(256)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    p = ctypes.c_void_p(a.data_ptr())
    rc = lib.matmul_launch_noalloc(native.handle, 8, 0, p, p, ctypes.c_void_p(out.data_ptr()), 2, 2, 2, stream,
                                   err, len(err))
    assert rc == 1 and err.value.decode().startswith("matmul_launch_noalloc: ")
