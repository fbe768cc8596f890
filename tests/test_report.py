"""The results.json (schema 3) report: row and file format on the CPU, one small
end-to-end report on the GPU (restates the reference's report contract,
src/main.py:91-103 and :184-196)."""

from __future__ import annotations

import csv
import json

import pytest

import report

REFERENCE_ROW_KEYS = ["backend", "execution_device", "precision", "input_dtype", "output_dtype", "mode", "m", "k",
                      "n", "median_ms", "p10_ms", "p90_ms", "tflops", "setup_ms", "kernel_config"]
ERROR_KEYS = ["max_abs_error", "arithmetic_max_abs_error", "max_tolerance_ratio", "arithmetic_reference",
              "roundoff_bound_max", "relative_frobenius_error", "arithmetic_relative_error",
              "quantization_relative_error"]


def test_parse_shape():
    assert report.parse_shape("1024") == (1024, 1024, 1024)
    assert report.parse_shape("16x8192x4096") == (16, 8192, 4096)
    assert report.parse_shape("31×33×65") == (31, 33, 65)
    for bad in ("0", "1x2", "4x-1x3"):
        with pytest.raises(ValueError):
            report.parse_shape(bad)


def test_result_row_keys_percentiles_and_tflops():
    errors = {key: 0.0 for key in ERROR_KEYS}
    row = report.result_row("tcgen05", "bf16", "device", (2, 3, 4), [4.0, 1.0, 2.0, 3.0], errors, 5.0, "cuda",
                            {"tile_m": 256})
    assert list(row)[:len(REFERENCE_ROW_KEYS)] == REFERENCE_ROW_KEYS
    assert row["input_dtype"] == "bfloat16" and row["output_dtype"] == "float32"
    assert row["median_ms"] == 2.5
    assert row["p10_ms"] == pytest.approx(1.3) and row["p90_ms"] == pytest.approx(3.7)
    assert row["tflops"] == pytest.approx(2 * 2 * 3 * 4 / (2.5 * 1e9))
    assert row["samples_ms"] == [4.0, 1.0, 2.0, 3.0]
    with pytest.raises(RuntimeError):
        report.result_row("ffma", "fp32", "device", (1, 1, 1), [1.0, float("nan")], errors, 0.0, "cuda", None)


def test_gamma_matches_the_reference_bound():
    assert report.gamma(4, 2.0 ** -23) == pytest.approx(4 * 2.0 ** -23 / (1 - 4 * 2.0 ** -23))
    assert report.gamma(2 ** 23, 2.0 ** -23) == float("inf")


def test_write_report_json_and_csv(tmp_path):
    errors = {key: 0.5 for key in ERROR_KEYS}
    rows = [report.result_row("ffma", "fp32", mode, (8, 8, 8), [1.0, 2.0], errors, 1.0, "cuda", {"a": 1})
            for mode in ("device", "resident")]
    rows[0]["gpu_checker_tolerance_ratio"] = 0.25     # a column only some rows have
    doc = {"schema_version": 3, "metadata": {"x": 1}, "measurements": rows, "unsupported_cases": []}
    report.write_report(doc, tmp_path / "out")
    loaded = json.loads((tmp_path / "out" / "results.json").read_text())
    assert loaded["schema_version"] == 3 and len(loaded["measurements"]) == 2
    with (tmp_path / "out" / "results.csv").open() as file:
        table = list(csv.DictReader(file))
    assert len(table) == 2 and "samples_ms" not in table[0]
    assert table[0]["gpu_checker_tolerance_ratio"] == "0.25" and table[1]["gpu_checker_tolerance_ratio"] == ""
    assert json.loads(table[0]["kernel_config"]) == {"a": 1}


def test_unsupported_backend_precisions():
    assert report.backend_supports("torch", "fp16")
    assert not report.backend_supports("ffma", "bf16")
    assert not report.backend_supports("tcgen05", "fp32")


@pytest.mark.gpu
def test_small_report_on_the_gpu(tmp_path):
    out = tmp_path / "results"
    report.main(["--sizes", "64", "33x65x17", "--warmup", "1", "--repeats", "3", "--output", str(out)])
    doc = json.loads((out / "results.json").read_text())
    assert doc["schema_version"] == 3
    assert doc["metadata"]["native_libraries"]["b200_matmul"]["abi"] == 3
    rows = doc["measurements"]
    # 2 shapes x (tcgen05: 3 precisions + ffma: 1 + torch: 4) x 3 modes
    assert len(rows) == 2 * 8 * 3
    for row in rows:
        assert set(REFERENCE_ROW_KEYS + ERROR_KEYS + ["samples_ms"]) <= set(row)
        assert row["max_tolerance_ratio"] <= 1.0
        if row["backend"] != "torch":
            assert row["gpu_checker_tolerance_ratio"] <= 1.0
            assert row["kernel_config"]["plan"]["kernel"]
    assert {(u["backend"], u["precision"]) for u in doc["unsupported_cases"]} == {
        ("tcgen05", "fp32"), ("ffma", "tf32"), ("ffma", "fp16"), ("ffma", "bf16")}
