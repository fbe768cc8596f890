"""bench.py's contract on the CPU: the reference arm's JSON line, rank handling
under torchrun (rank 0 alone prints), the warm-up floor and the ``--cases``
parser.  Nothing here needs a GPU."""

from __future__ import annotations

import json
import socket
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

import bench  # noqa: E402


def _json_lines(stdout: str) -> list[dict]:
    return [json.loads(line) for line in stdout.splitlines() if line.startswith("{")]


def _bench(*args: str, timeout: int = 600) -> subprocess.CompletedProcess:
    return subprocess.run([sys.executable, str(ROOT / "bench.py"), *args], capture_output=True, text=True,
                          timeout=timeout, cwd=ROOT)


def test_reference_arm_prints_the_contract_line():
    result = _bench("--impl", "reference", "--steps", "1", "--warmup", "3")
    assert result.returncode == 0, result.stderr[-2000:]
    lines = _json_lines(result.stdout)
    assert len(lines) == 1
    line = lines[0]
    assert line["impl"] == "reference"
    assert line["metric"] == bench.METRIC and line["unit"] == "TFLOP/s" and line["value"] > 0
    assert (line["n_gpus"], line["steps"], line["warmup"]) == (1, 1, 3)
    assert line["higher_is_better"] is True and line["vs_baseline"] is None
    baseline = line["cpu_baseline"]
    assert baseline["kind"] == "port" and baseline["cores"] >= 1 and baseline["value"] == line["value"]
    assert baseline["unit"] == line["unit"] and baseline["sample"]
    assert line["e2e"] == {"value": line["value"], "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}


def _free_port() -> int:
    with socket.socket() as sock:
        sock.bind(("127.0.0.1", 0))
        return sock.getsockname()[1]


def test_reference_arm_under_torchrun_prints_once():
    """Launched like the multi-GPU arm (one process per GPU), only rank 0 works and prints."""
    result = subprocess.run(
        [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2", "--master-addr",
         "127.0.0.1", "--master-port", str(_free_port()), str(ROOT / "bench.py"), "--impl", "reference",
         "--gpus", "2", "--steps", "1", "--warmup", "3"],
        capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert result.returncode == 0, result.stderr[-2000:]
    lines = _json_lines(result.stdout)
    assert len(lines) == 1
    assert lines[0]["impl"] == "reference" and lines[0]["n_gpus"] == 2 and lines[0]["scaling"] == "strong"


def test_fewer_than_three_warmup_steps_are_refused():
    result = _bench("--impl", "reference", "--steps", "1", "--warmup", "2", timeout=120)
    assert result.returncode != 0
    assert "warm-up" in result.stderr


def test_case_parser():
    assert bench.parse_case("4096x4096x4096:tf32") == (4096, 4096, 4096, "tf32", "uniform")
    assert bench.parse_case("16X8192x8192:bf16:normal") == (16, 8192, 8192, "bf16", "normal")
    for bad in ("4096x4096:bf16", "4096x4096x4096:int8", "0x1x1:fp32", "1x1x1:fp16:gaussian", "1x1x1"):
        with pytest.raises(SystemExit):
            bench.parse_case(bad)


def test_multi_gpu_defaults():
    """The driver's multi-GPU command uses the copy-engine broadcast with 2 SMs left
    to the one-element all-reduces; the NCCL broadcast keeps 8 for its kernels;
    an explicit --reserve-sms wins."""
    args = bench.parse_args(["--gpus", "8"])
    assert (args.broadcast, args.exchange, args.gather) == ("ce", "ce", "root")
    assert args.reserve_sms == 2
    assert args.workload == "rowshard32768" and args.steps == 20
    assert bench.parse_args(["--gpus", "8", "--broadcast", "nccl"]).reserve_sms == 8
    assert bench.parse_args(["--gpus", "8", "--reserve-sms", "0"]).reserve_sms == 0
    single = bench.parse_args([])
    assert single.workload == "square8192" and single.steps == 21 and single.warmup == 10
