"""The reference's CPU GEMM backends, restated (TEST AND CPU-BASELINE INFRASTRUCTURE ONLY).

Only ``bench.py``'s CPU-baseline leg and ``--impl reference`` arm call this;
the product never does.  It restates the two CPU backends of
chudinovAI/matrix-multiplication that time FP32 GEMM on the host:

* ``numpy_gemm``      -- ``src/benchmark_backends.py:223-226``: ``np.matmul(a, b, out=out)``
                         on FP32 row-major arrays with a reused output;
* ``torch_cpu_gemm``  -- ``src/benchmark_backends.py:229-235``: ``torch.mm(a, b, out=out)``.

Both use every host thread the BLAS library is given (the reference sets the
thread count through OMP/OPENBLAS/MKL variables before importing numpy,
``src/main.py:69-74``).
"""

from __future__ import annotations

import time

import numpy as np


def blas_threads() -> int:
    """Threads the BLAS behind numpy will use (threadpoolctl), else os.cpu_count()."""
    try:
        from threadpoolctl import threadpool_info

        counts = [info.get("num_threads", 0) for info in threadpool_info() if info.get("user_api") == "blas"]
        if counts:
            return int(max(counts))
    except Exception:
        pass
    import os

    return os.cpu_count() or 1


def numpy_gemm(a: np.ndarray, b: np.ndarray, out: np.ndarray) -> np.ndarray:
    """benchmark_backends.py:223-226."""
    return np.matmul(a, b, out=out)


def torch_cpu_gemm(a, b, out):
    """benchmark_backends.py:229-235."""
    import torch

    return torch.mm(a, b, out=out)


def time_numpy_slabs(a: np.ndarray, b: np.ndarray, rows: int, seconds: float, *, min_slabs: int = 1) -> dict:
    """Run ``a[i:i+rows] @ b`` over consecutive row slabs for about ``seconds``.

    Returns total flops, elapsed seconds and the number of slabs (the bounded
    sample that stands in for the full-size CPU GEMM).
    """
    m, k = a.shape
    n = b.shape[1]
    rows = max(1, min(rows, m))
    out = np.empty((rows, n), dtype=np.float32)
    numpy_gemm(a[:rows], b, out)                  # warm the BLAS threads
    slabs = 0
    flops = 0.0
    start = time.perf_counter()
    row = 0
    while True:
        stop = min(row + rows, m)
        numpy_gemm(a[row:stop], b, out[:stop - row])
        flops += 2.0 * (stop - row) * k * n
        slabs += 1
        row = 0 if stop >= m else stop
        elapsed = time.perf_counter() - start
        if slabs >= min_slabs and elapsed >= seconds:
            break
    return {"flops": flops, "seconds": elapsed, "slabs": slabs, "rows": rows}
