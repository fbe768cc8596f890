"""Parity of the B200 library with the CPU oracle, through the C-ABI (needs a B200).

Restates the reference's tests/test_matmul.py for this library's backends
(``tcgen05`` for TF32/FP16/BF16, ``ffma`` for FP32):

* every (backend, precision) on the reference shapes with inputs offset by
  one element (test_matmul.py:28-51), plus the ragged shapes of the benchmark
  configuration, tile-edge shapes and 16-byte-aligned shapes that take the
  TMA fast path, each run twice and verified by ``GemmReference``;
* a non-default stream and CUDA-graph capture (test_matmul.py:74-99);
* the exact TF32 RNE known answers (test_matmul.py:101-111 and
  test_triton_matmul.py:45-53) and FP16/BF16 ties through an identity B
  (test_metalmat.py:48-57, :108-117);
* contract, overlap, lifetime and invalid-device behaviour (test_matmul.py:113-199);
* large square and skinny shapes at benchmark sizes, checked on sampled rows;
* guard bands around the output (no write outside C) and the device status word.
"""

from __future__ import annotations

import ctypes
import gc
import weakref
from pathlib import Path

import numpy as np
import pytest
import torch

import precision_oracle as po
from precision import BACKEND_PRECISIONS, INPUT_DTYPES, PRECISIONS

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]
REFERENCE_SHAPES = ((1, 1, 1), (7, 13, 11), (35, 37, 67), (129, 35, 133), (2, 2049, 3))
RAGGED_SHAPES = ((31, 33, 65), (511, 257, 129), (513, 129, 577))
EDGE_SHAPES = ((128, 64, 256), (129, 65, 257), (255, 127, 255), (300, 1000, 520), (17, 65, 19), (3, 2049, 5))
ALIGNED_SHAPES = ((128, 64, 256), (256, 512, 512), (384, 192, 768), (1000, 1024, 1000), (640, 4096, 264),
                  # one shape per tcgen05 kernel choice: single-CTA 256-, 128-, 64-wide tiles, CTA pairs
                  (100, 64, 37888), (64, 128, 16384), (300, 96, 300), (2048, 128, 2048), (1024, 256, 4864),
                  # skinny: 16-row A boxes into 32-row stages, 16-deep ring
                  (16, 512, 8192), (32, 1024, 4096))
PLANS = [(backend, precision) for backend in ("tcgen05", "ffma") for precision in BACKEND_PRECISIONS[backend]]


def _dtype(precision):
    return getattr(torch, INPUT_DTYPES[precision])


def _offset_matrix(rows, cols, dtype, offset=1):
    """A contiguous rows x cols view whose base is `offset` elements past an allocation."""
    return torch.empty(rows * cols + offset, dtype=dtype, device="cuda")[offset:].view(rows, cols)


def _run_and_verify(native, backend, precision, a_np, b_np, *, offset, runs=2, baseline_c=2.0):
    m, k = a_np.shape
    n = b_np.shape[1]
    reference = po.GemmReference(a_np, b_np, precision)
    dtype = _dtype(precision)
    if offset:
        a = _offset_matrix(m, k, dtype)
        b = _offset_matrix(k, n, dtype)
        out = _offset_matrix(m, n, torch.float32)
    else:
        a = torch.empty((m, k), dtype=dtype, device="cuda")
        b = torch.empty((k, n), dtype=dtype, device="cuda")
        out = torch.empty((m, n), dtype=torch.float32, device="cuda")
    a.copy_(torch.from_numpy(a_np))
    b.copy_(torch.from_numpy(b_np))
    run = native.prepare(backend, a, b, out, precision=precision)
    for _ in range(runs):
        out.fill_(float("nan"))
        run()
        torch.cuda.current_stream().synchronize()
        actual = out.cpu().numpy()
        report = reference.verify(actual, f"{backend}/{precision} {m}x{k}x{n}")
    ratio = po.baseline_bound_ratio(a_np, b_np, actual, precision, c=baseline_c)
    assert ratio <= 1.0, f"outside c*K*u*sum|a||b| with c={baseline_c}: ratio {ratio}"
    return report


@pytest.mark.parametrize("backend,precision", PLANS)
@pytest.mark.parametrize("shape", REFERENCE_SHAPES + RAGGED_SHAPES + EDGE_SHAPES)
def test_offset_operands_against_fp64_oracle(native, backend, precision, shape):
    m, k, n = shape
    rng = np.random.default_rng(923 + m + k + n)
    a_np = rng.standard_normal((m, k)).astype(np.float32)
    b_np = rng.standard_normal((k, n)).astype(np.float32)
    _run_and_verify(native, backend, precision, a_np, b_np, offset=True)


@pytest.mark.parametrize("backend,precision", PLANS)
@pytest.mark.parametrize("shape", ALIGNED_SHAPES + RAGGED_SHAPES)
def test_aligned_operands_against_fp64_oracle(native, backend, precision, shape):
    m, k, n = shape
    a_np = po.seeded_uniform((m, k), seed=m * 7 + k)
    b_np = po.seeded_uniform((k, n), seed=n * 11 + k)
    _run_and_verify(native, backend, precision, a_np, b_np, offset=False)


@pytest.mark.parametrize("backend,precision", PLANS)
def test_prepared_nondefault_stream_and_graph(native, backend, precision):
    rng = np.random.default_rng(14)
    a_np = rng.standard_normal((7, 13)).astype(np.float32)
    b_np = rng.standard_normal((13, 11)).astype(np.float32)
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        a = torch.from_numpy(a_np).to(device="cuda", dtype=_dtype(precision))
        b = torch.from_numpy(b_np).to(device="cuda", dtype=_dtype(precision))
        out = torch.empty((7, 11), dtype=torch.float32, device="cuda")
        run = native.prepare(backend, a, b, out, precision=precision)
        run()
        stream.synchronize()
        out.fill_(float("nan"))
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            run()
        graph.replay()
        stream.synchronize()
    po.GemmReference(a_np, b_np, precision).verify(out.cpu().numpy(), f"{backend}/graph")
    del graph


# Tensor-core shapes whose plans split K over clusters of 2, 4 and 8 CTAs (long K
# against few output tiles), including a C that TMA cannot store (n % 4 != 0), an
# unaligned K and m < 128.
TC_SPLIT_SHAPES = ((1024, 4096, 1024), (512, 8192, 512), (96, 4096, 2048), (200, 3000, 300), (130, 4099, 258),
                   (65, 2000, 70))


SKINNY_SPLIT_SHAPES = ((16, 8192, 1024), (48, 4096, 2048), (5, 3000, 260), (64, 2048, 8192), (32, 1024, 4096))


def test_skinny_plans_split_k(native):
    assert native.plan("tcgen05", 16, 8192, 8192, precision="bf16") == {
        "kernel": "tc_skinny", "tile_m": 16, "tile_n": 128, "splits": 2}
    splits = {native.plan("tcgen05", *shape, precision=p)["splits"]
              for shape in SKINNY_SPLIT_SHAPES for p in ("tf32", "fp16", "bf16")}
    assert splits >= {2, 4, 8}


@pytest.mark.parametrize("precision", ("tf32", "fp16", "bf16"))
@pytest.mark.parametrize("shape", SKINNY_SPLIT_SHAPES)
def test_skinny_split_k_against_fp64_oracle(native, precision, shape):
    m, k, n = shape
    a_np = po.seeded_uniform((m, k), seed=17 * m + k)
    b_np = po.seeded_uniform((k, n), seed=19 * n + k)
    _run_and_verify(native, "tcgen05", precision, a_np, b_np, offset=False)


def test_tcgen05_plans_split_k(native):
    splits = set()
    for precision in ("tf32", "fp16", "bf16"):
        for shape in TC_SPLIT_SHAPES:
            plan = native.plan("tcgen05", *shape, precision=precision)
            m, k, n = shape
            if precision == "tf32" and m * k * n <= 2 ** 25:
                assert plan["kernel"] == "ffma_tf32_rne"      # small TF32 problems run on the FFMA pipe
                continue
            assert plan["kernel"] == "tc_single"
            splits.add(plan["splits"])
    assert splits >= {2, 4, 8}
    assert native.plan("tcgen05", 8192, 8192, 8192, precision="bf16")["kernel"] == "tc2_pair"


# Shapes the launch plan gives the 256 x 512 CTA-pair tile (one accumulator freed
# in column halves, deferred upper-half MMAs at both ends of every tile).
WIDE_PAIR_SHAPES = ((3001, 2048, 5003), (2048, 1024, 4096), (1537, 777, 3001))


def test_wide_pair_plans(native):
    for m, k, n in WIDE_PAIR_SHAPES + ((8192, 8192, 8192), (4096, 14336, 4096)):
        for precision in ("tf32", "fp16", "bf16"):
            if (m, k, n) == (1537, 777, 3001) and precision != "tf32":
                continue
            plan = native.plan("tcgen05", m, k, n, precision=precision)
            assert (plan["kernel"], plan["tile_m"], plan["tile_n"]) == ("tc2_pair", 256, 512), (m, k, n, plan)


@pytest.mark.parametrize("precision", ("tf32", "fp16", "bf16"))
@pytest.mark.parametrize("shape", WIDE_PAIR_SHAPES)
def test_wide_pair_against_fp64_oracle(native, precision, shape):
    m, k, n = shape
    a_np = po.seeded_uniform((m, k), seed=17 * m + k)
    b_np = po.seeded_uniform((k, n), seed=19 * n + k)
    _run_and_verify(native, "tcgen05", precision, a_np, b_np, offset=shape[1] % 2 == 1, runs=1)


@pytest.mark.parametrize("precision", ("tf32", "fp16", "bf16"))
@pytest.mark.parametrize("shape", TC_SPLIT_SHAPES)
def test_tcgen05_split_k_against_fp64_oracle(native, precision, shape):
    m, k, n = shape
    a_np = po.seeded_uniform((m, k), seed=11 * m + k)
    b_np = po.seeded_uniform((k, n), seed=13 * n + k)
    _run_and_verify(native, "tcgen05", precision, a_np, b_np, offset=False)


@pytest.mark.parametrize("shape,sms", (((2048, 1024, 3072), 40), ((4096, 2048, 4096), 132)))
def test_sm_limit_bounds_the_launch_and_keeps_results(native, shape, sms):
    """132 SMs is what the row-sharded multi-GPU step leaves the GEMM (16 reserved for
    NCCL); that shape runs on the 256 x 512 pair tile."""
    m, k, n = shape
    full = native.plan("tcgen05", m, k, n, precision="bf16")
    a_np = po.seeded_uniform((m, k), 21)
    b_np = po.seeded_uniform((k, n), 22)
    try:
        native.set_sm_limit(sms)
        limited = native.plan("tcgen05", m, k, n, precision="bf16")
        assert limited["ctas"] <= sms < full["ctas"]
        if sms == 132:
            assert (limited["kernel"], limited["tile_n"]) == ("tc2_pair", 512)
        _run_and_verify(native, "tcgen05", "bf16", a_np, b_np, offset=False, runs=1)
        with pytest.raises(RuntimeError):
            native.set_sm_limit(1)
    finally:
        native.set_sm_limit(0)
    assert native.plan("tcgen05", m, k, n, precision="bf16") == full


def test_tcgen05_split_k_is_deterministic_and_graph_capturable(native):
    m, k, n = 512, 8192, 512
    assert native.plan("tcgen05", m, k, n, precision="bf16")["splits"] > 1
    a = torch.from_numpy(po.seeded_uniform((m, k), 3)).cuda().to(torch.bfloat16)
    b = torch.from_numpy(po.seeded_uniform((k, n), 4)).cuda().to(torch.bfloat16)
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        first = torch.empty((m, n), device="cuda")
        second = torch.full((m, n), float("nan"), device="cuda")
        native.prepare("tcgen05", a, b, first, precision="bf16")()
        run = native.prepare("tcgen05", a, b, second, precision="bf16")
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            run()
        graph.replay()
        stream.synchronize()
    assert torch.equal(first, second)
    del graph


# Aligned FP32 shapes whose launch plans (matmul_plan) cover both FFMA tiles and
# K splits of 1, 2, 4 and 8 cluster CTAs, including splits that get no K tiles
# (32 x 144 x 32: 9 K tiles over 8 CTAs).
FFMA_PLAN_SHAPES = ((64, 64, 64), (128, 128, 128), (32, 144, 32), (100, 3000, 200), (384, 2048, 640),
                    (768, 768, 768), (1024, 64, 1024), (1536, 256, 1536), (1024, 1024, 1024),
                    (640, 1024, 832), (2048, 512, 2048), (1200, 64, 2400), (260, 2052, 196),
                    (1408, 512, 1408), (512, 2048, 896))


def test_ffma_plans_cover_every_tile_and_split(native):
    plans = {shape: native.plan("ffma", *shape) for shape in FFMA_PLAN_SHAPES}
    assert {p["kernel"] for p in plans.values()} == {"ffma_async"}
    assert {(p["tile_m"], p["tile_n"]) for p in plans.values()} == {(128, 128), (32, 32)}
    assert {p["splits"] for p in plans.values()} == {1, 2, 4, 8}
    assert {p["splits"] for p in plans.values() if p["tile_m"] == 128} >= {1, 2, 4}
    assert plans[(32, 144, 32)]["splits"] == 8
    ragged = native.plan("ffma", 31, 33, 65)
    assert ragged["kernel"] == "ffma_async" and ragged["vector_loads_if_aligned"] is False


@pytest.mark.parametrize("shape", FFMA_PLAN_SHAPES)
def test_ffma_split_k_plans_against_fp64_oracle(native, shape):
    m, k, n = shape
    a_np = po.seeded_uniform((m, k), seed=3 * m + k)
    b_np = po.seeded_uniform((k, n), seed=5 * n + k)
    report = _run_and_verify(native, "ffma", "fp32", a_np, b_np, offset=False)
    assert report["max_tolerance_ratio"] <= 1.0


def test_ffma_split_k_is_deterministic_and_graph_capturable(native):
    m, k, n = 100, 3000, 200
    assert native.plan("ffma", m, k, n)["splits"] > 1
    a = torch.from_numpy(po.seeded_uniform((m, k), 1)).cuda()
    b = torch.from_numpy(po.seeded_uniform((k, n), 2)).cuda()
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        first = torch.empty((m, n), device="cuda")
        second = torch.full((m, n), float("nan"), device="cuda")
        native.prepare("ffma", a, b, first, precision="fp32")()
        run = native.prepare("ffma", a, b, second, precision="fp32")
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            run()
        graph.replay()
        stream.synchronize()
    assert torch.equal(first, second)
    del graph


@pytest.mark.parametrize("shape", ((256, 512, 512), (129, 65, 257)))
@pytest.mark.parametrize("precision", ("tf32", "bf16"))
def test_graph_of_ten_launches_replays_correctly(native, precision, shape):
    """The benchmark's capture pattern (10 launches per graph), including the
    scratch-allocating paths (TF32 rounding, unaligned repacking)."""
    m, k, n = shape
    a_np = po.seeded_uniform((m, k), 5)
    b_np = po.seeded_uniform((k, n), 6)
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        a = torch.from_numpy(a_np).to(device="cuda", dtype=_dtype(precision))
        b = torch.from_numpy(b_np).to(device="cuda", dtype=_dtype(precision))
        out = torch.empty((m, n), dtype=torch.float32, device="cuda")
        run = native.prepare("tcgen05", a, b, out, precision=precision)
        run()
        stream.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            for _ in range(10):
                run()
        for _ in range(3):
            out.fill_(float("nan"))
            graph.replay()
        stream.synchronize()
    po.GemmReference(a_np, b_np, precision).verify(out.cpu().numpy(), "graph x10")
    del graph


@pytest.mark.parametrize("rows", (1, 4096))
def test_tf32_rounds_halfway_to_even(native, rows):
    """Bit-exact known answers: reference test_matmul.py:101-111 and test_triton_matmul.py:45-53.

    One row runs on the small-problem FFMA path (K tiles rounded in shared memory),
    4096 rows x 1024 columns on the tensor cores (operands rounded by the TMA loads of
    their TFLOAT32 tensor maps)."""
    bits = np.array([0x3f801000, 0x3f803000, 0x3f800fff, 0x3f801001,
                     0xbf801000, 0xbf803000, 0xbf800fff, 0xbf801001], dtype=np.uint32)
    values = np.tile(bits.view(np.float32).reshape(1, -1), (rows, 1 if rows == 1 else 128))
    size = values.shape[1]
    plan = native.plan("tcgen05", rows, size, size, precision="tf32")
    assert (plan["kernel"] == "ffma_tf32_rne") == (rows == 1)
    a = torch.from_numpy(values).cuda()
    b = torch.eye(size, dtype=torch.float32, device="cuda")
    out = torch.empty((rows, size), dtype=torch.float32, device="cuda")
    native.prepare("tcgen05", a, b, out, precision="tf32")()
    np.testing.assert_array_equal(out.cpu().numpy(), po.quantize_inputs(values, "tf32"))
    if rows == 1:
        expected = po.reference_product(values, np.eye(size, dtype=np.float32), "tf32")
        np.testing.assert_array_equal(out.cpu().numpy(), expected)


@pytest.mark.parametrize("precision", ("fp16", "bf16"))
def test_half_formats_round_ties_to_even(native, precision):
    """Identity-B known answers (reference test_metalmat.py:48-57, :108-117): the
    device input is produced by the library's own FP32 -> FP16/BF16 conversion."""
    step = 2.0 ** (-10 if precision == "fp16" else -7)
    values = np.array([[1 + step / 2, 1 + 3 * step / 2, -1 - step / 2, -1 - 3 * step / 2,
                        2.0**-24, 2.0**-25]], dtype=np.float32)
    source = torch.from_numpy(values).cuda()
    a = torch.empty(values.shape, dtype=_dtype(precision), device="cuda")
    native.convert(source, a, precision)
    eye = torch.eye(values.shape[1], dtype=torch.float32, device="cuda")
    b = torch.empty(eye.shape, dtype=_dtype(precision), device="cuda")
    native.convert(eye, b, precision)
    out = torch.empty(values.shape, dtype=torch.float32, device="cuda")
    native.prepare("tcgen05", a, b, out, precision=precision)()
    expected = po.reference_product(values, np.eye(values.shape[1], dtype=np.float32), precision)
    np.testing.assert_array_equal(out.cpu().numpy(), expected.astype(np.float32))


@pytest.mark.parametrize("precision", PRECISIONS)
def test_device_conversion_matches_oracle_bit_for_bit(native, golden, precision):
    probe = golden["probe"]
    finite = probe[np.isfinite(probe) & (np.abs(probe) < 6e4)]
    src = torch.from_numpy(np.ascontiguousarray(finite)).cuda()
    dst = torch.empty(src.shape, dtype=_dtype(precision), device="cuda")
    native.convert(src, dst, precision)
    got = dst.float().cpu().numpy()
    np.testing.assert_array_equal(got.view(np.uint32), po.quantize_inputs(finite, precision).view(np.uint32))


def test_invalid_tensor_contracts(native):
    a = torch.ones((2, 3), dtype=torch.float32, device="cuda")
    b = torch.ones((3, 4), dtype=torch.float32, device="cuda")
    out = torch.empty((2, 4), dtype=torch.float32, device="cuda")
    cases = [
        ("unknown", a, b, out, ValueError),
        ("ffma", None, b, out, TypeError),
        ("ffma", a.flatten(), b, out, ValueError),
        ("ffma", a.double(), b, out, TypeError),
        ("ffma", a.cpu(), b, out, ValueError),
        ("ffma", torch.ones((3, 2), device="cuda").T, b, out, ValueError),
        ("ffma", a, b[:2], out, ValueError),
        ("ffma", a, b, out[:, :3].contiguous(), ValueError),
        ("ffma", a[:0], b, out[:0], ValueError),
        ("wmma", a, b, out, ValueError),
    ]
    for backend, left, right, result, error in cases:
        with pytest.raises(error):
            native.prepare(backend, left, right, result)
    if torch.cuda.device_count() > 1:
        with pytest.raises(ValueError):
            native.prepare("ffma", a.to("cuda:1"), b, out)


def test_precision_contracts(native):
    a = torch.ones((2, 3), dtype=torch.float32, device="cuda")
    b = torch.ones((3, 4), dtype=torch.float32, device="cuda")
    out = torch.empty((2, 4), dtype=torch.float32, device="cuda")
    with pytest.raises(ValueError):
        native.prepare("tcgen05", a, b, out, precision="invalid")
    for precision in ("tf32", "fp16", "bf16"):
        with pytest.raises(ValueError):
            native.prepare("ffma", a.to(_dtype(precision)), b.to(_dtype(precision)), out, precision=precision)
    with pytest.raises(ValueError):
        native.prepare("tcgen05", a, b, out, precision="fp32")
    for precision in ("fp16", "bf16"):
        with pytest.raises(TypeError):
            native.prepare("tcgen05", a, b, out, precision=precision)
    with pytest.raises(TypeError):
        native.prepare("ffma", a, b, out.half(), precision="fp32")


def test_native_launch_rejects_bad_arguments(native):
    """The C entry point itself rejects bad ids and sizes (matmul.cu:354-367)."""
    lib = native.library
    a = torch.ones((2, 2), device="cuda")
    out = torch.empty((2, 2), device="cuda")
    err = ctypes.create_string_buffer(256)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    p = ctypes.c_void_p(a.data_ptr())
    o = ctypes.c_void_p(out.data_ptr())
    for impl, prec, m, k, n in ((7, 0, 2, 2, 2), (8, 3, 2, 2, 2), (6, 3, 2, 2, 2), (8, 0, 0, 2, 2),
                                (8, 0, 2, -1, 2), (99, 0, 2, 2, 2)):
        assert lib.matmul_launch(native.handle, impl, prec, p, p, o, m, k, n, stream, err, len(err)) == 1
        assert err.value.decode().startswith("matmul_launch: ")
    odd = ctypes.c_void_p(a.data_ptr() + 1)
    assert lib.matmul_launch(native.handle, 8, 0, odd, p, o, 1, 1, 1, stream, err, len(err)) == 1
    assert lib.matmul_launch(native.handle, 8, 0, None, p, o, 1, 1, 1, stream, err, len(err)) == 1


def test_partial_overlap_rejected_but_disjoint_storage_works(native):
    storage = torch.arange(12, dtype=torch.float32, device="cuda")
    first = storage[:4].view(2, 2)
    overlapping = storage[1:5].view(2, 2)
    disjoint = storage[4:8].view(2, 2)
    independent = torch.ones((2, 2), dtype=torch.float32, device="cuda")
    with pytest.raises(ValueError):
        native.prepare("ffma", first, independent, overlapping)
    with pytest.raises(ValueError):
        native.prepare("ffma", independent, first, overlapping)
    native.prepare("ffma", first, independent, disjoint)()
    torch.cuda.synchronize()
    np.testing.assert_array_equal(disjoint.cpu().numpy(), [[1, 1], [5, 5]])


def test_prepared_operation_retains_tensors_and_rejects_closed_context(native):
    a = torch.ones((2, 2), dtype=torch.bfloat16, device="cuda")
    b = torch.ones((2, 2), dtype=torch.bfloat16, device="cuda")
    out = torch.empty((2, 2), dtype=torch.float32, device="cuda")
    references = [weakref.ref(tensor) for tensor in (a, b, out)]
    run = native.prepare("tcgen05", a, b, out, precision="bf16")
    del a, b, out
    gc.collect()
    run()
    torch.cuda.synchronize()
    np.testing.assert_array_equal(references[2]().cpu().numpy(), [[2, 2], [2, 2]])
    assert native.device_status() == 0
    native.close()
    native.close()
    with pytest.raises(RuntimeError):
        run()
    with pytest.raises(RuntimeError):
        native.prepare("ffma", None, None, None)
    with pytest.raises(RuntimeError):
        native.configuration("ffma")
    del run
    gc.collect()
    assert all(reference() is None for reference in references)


def test_invalid_device_does_not_poison_a_later_valid_launch(native, library_path):
    from gpumat import NativeMatmul

    with pytest.raises(RuntimeError):
        NativeMatmul(library_path, device=torch.cuda.device_count())
    a = torch.tensor([[2.0, -3.0]], device="cuda")
    b = torch.tensor([[4.0], [5.0]], device="cuda")
    out = torch.empty((1, 1), device="cuda")
    native.prepare("ffma", a, b, out)()
    torch.cuda.synchronize()
    np.testing.assert_array_equal(out.cpu().numpy(), [[-7.0]])


@pytest.mark.parametrize("backend,precision", PLANS)
@pytest.mark.parametrize("offset", (0, 1))
def test_no_write_outside_the_output(native, backend, precision, offset):
    """Canary values before and after C survive every launch (partial tiles included)."""
    m, k, n = 133, 70, 261
    guard = 4096
    a_np = po.seeded_uniform((m, k), 1)
    b_np = po.seeded_uniform((k, n), 2)
    dtype = _dtype(precision)
    a = torch.from_numpy(a_np).to(device="cuda", dtype=dtype)
    b = torch.from_numpy(b_np).to(device="cuda", dtype=dtype)
    storage = torch.full((guard + m * n + offset + guard,), 12345.0, dtype=torch.float32, device="cuda")
    out = storage[guard + offset:guard + offset + m * n].view(m, n)
    native.prepare(backend, a, b, out, precision=precision)()
    torch.cuda.synchronize()
    host = storage.cpu().numpy()
    assert np.all(host[:guard + offset] == 12345.0)
    assert np.all(host[guard + offset + m * n:] == 12345.0)
    po.GemmReference(a_np, b_np, precision).verify(out.cpu().numpy(), "guarded")


def _sampled_check(native, backend, precision, m, k, n, *, generator="uniform", rows=12):
    if generator == "uniform":
        a_np = po.seeded_uniform((m, k), 100 + m)
        b_np = po.seeded_uniform((k, n), 200 + n)
    else:
        a_np = po.seeded_normal((m, k), 100 + m, scale=k ** -0.5)
        b_np = po.seeded_normal((k, n), 200 + n, scale=k ** -0.5)
    dtype = _dtype(precision)
    a = torch.from_numpy(a_np).to(device="cuda", dtype=dtype)
    b = torch.from_numpy(b_np).to(device="cuda", dtype=dtype)
    out = torch.full((m, n), float("nan"), dtype=torch.float32, device="cuda")
    native.prepare(backend, a, b, out, precision=precision)()
    torch.cuda.synchronize()
    picked = np.unique(np.concatenate([[0, m - 1], np.random.default_rng(m).integers(0, m, rows)]))
    reference = po.sampled_reference(a_np, b_np, precision, picked)
    sampled = out[torch.from_numpy(picked).cuda()].cpu().numpy()
    reference.verify(sampled, f"{backend}/{precision} {m}x{k}x{n} sampled rows")
    assert torch.isfinite(out).all().item()
    ratio = po.baseline_bound_ratio(a_np[picked], b_np, sampled, precision, c=2.0)
    assert ratio <= 1.0
    return out


@pytest.mark.parametrize("precision", ("tf32", "fp16", "bf16"))
def test_large_square_tcgen05_sampled(native, precision):
    _sampled_check(native, "tcgen05", precision, 4096, 4096, 4096)


def test_large_square_ffma_sampled(native):
    _sampled_check(native, "ffma", "fp32", 2048, 2048, 2048)


@pytest.mark.parametrize("shape", ((8192, 8192, 8192), (16, 8192, 8192), (4096, 14336, 4096)))
@pytest.mark.parametrize("precision", ("fp16", "bf16"))
def test_benchmark_shapes_sampled(native, precision, shape):
    _sampled_check(native, "tcgen05", precision, *shape, generator="normal", rows=8)


def test_bf16_8192_full_output_checksum(native):
    """Size-independent check at 8192^3: the sum of C equals (1^T A)(B 1)
    computed in FP64 from the BF16-rounded inputs."""
    m = k = n = 8192
    a_np = po.seeded_normal((m, k), 7, scale=k ** -0.5)
    b_np = po.seeded_normal((k, n), 8, scale=k ** -0.5)
    a = torch.from_numpy(a_np).to(device="cuda", dtype=torch.bfloat16)
    b = torch.from_numpy(b_np).to(device="cuda", dtype=torch.bfloat16)
    out = torch.empty((m, n), dtype=torch.float32, device="cuda")
    native.prepare("tcgen05", a, b, out, precision="bf16")()
    torch.cuda.synchronize()
    qa = po.quantize_inputs(a_np, "bf16").astype(np.float64)
    qb = po.quantize_inputs(b_np, "bf16").astype(np.float64)
    expected = float(qa.sum(axis=0) @ qb.sum(axis=1))
    got = float(out.double().sum().item())
    magnitude = float(np.abs(qa).sum(axis=0) @ np.abs(qb).sum(axis=1))
    assert abs(got - expected) <= 1e-6 * magnitude + 1e-3


def test_reference_library_agrees(native):
    """Cross-check against the reference's own CUDA library built for sm_100a
    (oracle/_ref/matmul.so): its cuBLAS BF16 path and its wmma kernel."""
    path = ROOT / "oracle" / "_ref" / "matmul.so"
    if not path.exists():
        pytest.skip("reference library not built (make -C oracle ref)")
    lib = ctypes.CDLL(str(path))
    lib.matmul_create.restype = ctypes.c_void_p
    lib.matmul_create.argtypes = [ctypes.c_int, ctypes.c_char_p, ctypes.c_size_t]
    lib.matmul_launch.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p,
                                  ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p,
                                  ctypes.c_char_p, ctypes.c_size_t]
    lib.matmul_destroy.argtypes = [ctypes.c_void_p, ctypes.c_char_p, ctypes.c_size_t]
    err = ctypes.create_string_buffer(1024)
    ctx = lib.matmul_create(0, err, len(err))
    assert ctx, err.value
    m, k, n = 513, 129, 577
    a_np = po.seeded_uniform((m, k), 31)
    b_np = po.seeded_uniform((k, n), 32)
    a = torch.from_numpy(a_np).to(device="cuda", dtype=torch.bfloat16)
    b = torch.from_numpy(b_np).to(device="cuda", dtype=torch.bfloat16)
    ours = torch.empty((m, n), dtype=torch.float32, device="cuda")
    native.prepare("tcgen05", a, b, ours, precision="bf16")()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    reference = po.GemmReference(a_np, b_np, "bf16")
    for implementation in (2, 6):        # cublas, wmma
        theirs = torch.empty((m, n), dtype=torch.float32, device="cuda")
        rc = lib.matmul_launch(ctx, implementation, 3, ctypes.c_void_p(a.data_ptr()), ctypes.c_void_p(b.data_ptr()),
                               ctypes.c_void_p(theirs.data_ptr()), m, k, n, stream, err, len(err))
        assert rc == 0, err.value
        torch.cuda.synchronize()
        reference.verify(theirs.cpu().numpy(), f"reference impl {implementation}")
        difference = (ours - theirs).abs().max().item()
        assert difference <= 2 * float(reference.roundoff_bound.max()) + 1e-3
    reference.verify(ours.cpu().numpy(), "tcgen05")
    lib.matmul_destroy(ctx, err, len(err))


@pytest.mark.parametrize("precision,chunks,tail", [("bf16", 4, 1), ("bf16", 3, 4), ("tf32", 3, 2), ("fp32", 2, 1),
                                                   ("fp16", 1, 1)])
def test_host_to_host_pipeline(native, precision, chunks, tail):
    """end_to_end.HostMatmul: FP32 host inputs, on-device conversion, chunked GEMM
    and overlapped copies give the oracle's answer in a pinned host buffer."""
    from end_to_end import HostMatmul

    m, k, n = 1000, 384, 520
    a_np = po.seeded_uniform((m, k), 41)
    b_np = po.seeded_uniform((k, n), 42)
    host_gemm = HostMatmul(native, m, k, n, precision, chunks=chunks, tail_chunks=tail)
    assert [r for r in host_gemm.ranges if r[1] <= r[0]] == [] and host_gemm.ranges[-1][1] == m
    assert len(host_gemm.ranges) == chunks - 1 + tail
    a = torch.from_numpy(a_np).pin_memory()
    b = torch.from_numpy(b_np).pin_memory()
    c = torch.full((m, n), float("nan"), dtype=torch.float32).pin_memory()
    for _ in range(2):
        host_gemm(a, b, c)
        po.GemmReference(a_np, b_np, precision).verify(c.numpy(), f"host pipeline {precision}")
