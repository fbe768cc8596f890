"""Build the B200 GEMM library (the equivalent of the reference's ``make cuda``).

    python matrix-multiplication_b200/build.py [--verbose-ptxas]

Compiles ``csrc/matmul_b200.cu`` for sm_100a only into ``build/b200_matmul.so``
at the repository root (the same place relative to the loader as the
reference's ``build/matmul.so``).  The CUDA runtime is linked statically and
the driver API is reached through ``cudaGetDriverEntryPoint``, so the library
loads on a machine without a GPU driver (it then fails cleanly in
``matmul_create``).
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

PACKAGE = Path(__file__).resolve().parent
ROOT = PACKAGE.parent
SOURCE = PACKAGE / "csrc" / "matmul_b200.cu"
HEADERS = sorted((PACKAGE / "csrc").glob("*.cuh")) + [ROOT / "include" / "b200_matmul.h"]
OUTPUT = ROOT / "build" / "b200_matmul.so"
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    candidate = Path(home) / "bin" / "nvcc"
    return str(candidate) if candidate.exists() else (shutil.which("nvcc") or "nvcc")


def command(output: Path = OUTPUT, verbose_ptxas: bool = False) -> list[str]:
    cmd = [nvcc(), "-O3", "-std=c++17", *ARCH_FLAGS, "-lineinfo", "-shared", "-Xcompiler", "-fPIC",
           "-cudart", "static", "-I", str(ROOT / "include"), "-o", str(output), str(SOURCE)]
    if verbose_ptxas:
        cmd[1:1] = ["-Xptxas", "-v"]
    return cmd


def up_to_date(output: Path = OUTPUT) -> bool:
    if not output.exists():
        return False
    built = output.stat().st_mtime
    return all(path.stat().st_mtime <= built for path in [SOURCE, *HEADERS, Path(__file__)])


def build(force: bool = False, verbose_ptxas: bool = False, output: Path = OUTPUT) -> Path:
    """Compile the library unless it is newer than every source; return its path."""
    if not force and not verbose_ptxas and up_to_date(output):
        return output
    output.parent.mkdir(parents=True, exist_ok=True)
    tmp = output.with_suffix(".so.tmp")
    result = subprocess.run(command(tmp, verbose_ptxas), capture_output=True, text=True)
    if result.returncode != 0:
        raise RuntimeError(f"nvcc failed ({result.returncode}):\n{result.stdout}\n{result.stderr}")
    if verbose_ptxas:
        print(result.stderr, file=sys.stderr)
    os.replace(tmp, output)
    return output


def main() -> int:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--force", action="store_true")
    parser.add_argument("--verbose-ptxas", action="store_true")
    args = parser.parse_args()
    path = build(force=args.force, verbose_ptxas=args.verbose_ptxas)
    print(path)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
