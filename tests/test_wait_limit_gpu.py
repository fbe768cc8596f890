"""Failure detection on the GPU without a GPU fault (needs a B200).

The tensor-core kernels and the TMA-staged FFMA kernel bound every mbarrier wait.  ``matmul_set_wait_limit``
shortens the progress waits (a stage to land, an accumulator to fill or to be
read) to 1 ns, so that the first one that is not already complete runs out.
Each test then checks, for one kernel family picked through ``matmul_plan``:

* the launch returns and the device status word reports a progress timeout
  (and no drain timeout: copies and MMAs already issued always finish);
* the output holds NaN wherever the kernel did not finish, so the reference's
  FP64 check (``GemmReference.verify``) fails instead of passing over stale
  values;
* the context stays usable: with the default limit restored, the same
  prepared launch gives the oracle's answer and the status word stays 0
  (which also shows that the timed-out kernel released its tensor memory, or
  the next kernel could not have allocated any).

The reference's kernels have no waits that can run out; its error convention
is src/matmul.cu:36-47 (return codes) and :475-478 (launch errors).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import precision_oracle as po
from precision import INPUT_DTYPES

pytestmark = pytest.mark.gpu

LOAD, MMA, EPILOGUE, DRAIN = 1, 2, 4, 8

# family -> (precision, candidate shapes); the first candidate whose plan matches is
# used.  The tensor-core shapes have long K loops, so their first accumulator wait
# lasts far longer than one poll; with a 1 ns limit the waits poll once without
# suspending, so even the FFMA kernel's wait for its first stage runs out.
FAMILIES = {
    "single_cta": ("bf16", ((512, 4096, 4096), (1024, 4096, 2048), (2048, 4096, 1024))),
    "single_cta_split_k": ("bf16", ((512, 8192, 512), (1024, 16384, 1024), (512, 16384, 512))),
    "pair_256": ("bf16", ((2048, 8192, 2048), (2048, 16384, 2048), (2048, 4096, 2048))),
    "pair_512": ("bf16", ((2048, 8192, 4096), (4096, 8192, 4096), (3072, 4096, 3072))),
    "skinny": ("fp16", ((64, 4096, 32768), (48, 4096, 65536), (32, 8192, 65536))),
    "skinny_split_k": ("bf16", ((16, 8192, 8192), (16, 16384, 4096), (48, 8192, 2048))),
    "tf32_in_place": ("tf32", ((1024, 8192, 1024), (2048, 4096, 2048), (512, 8192, 512))),
    # The FFMA kernel's 128 x 128 tile with TMA-staged (16-byte aligned) operands.
    "ffma_tma": ("fp32", ((2048, 2048, 2048), (4096, 1024, 4096), (1536, 4096, 1536))),
    "ffma_tma_split_k": ("fp32", ((1024, 1024, 1024), (640, 1024, 832), (512, 2048, 896), (1408, 512, 1408),
                                  (1536, 256, 1536), (2048, 512, 2048))),
}


def _family_of(plan: dict) -> set[str]:
    kernel, splits = plan["kernel"], plan.get("splits", 1)
    names = set()
    if kernel == "tc_single":
        names.add("single_cta" if splits == 1 else "single_cta_split_k")
    elif kernel == "tc2_pair":
        names.add("pair_512" if plan["tile_n"] == 512 else "pair_256")
    elif kernel == "tc_skinny":
        names.add("skinny" if splits == 1 else "skinny_split_k")
    elif kernel == "ffma_async" and plan["tile_m"] == 128:
        names.add("ffma_tma" if splits == 1 else "ffma_tma_split_k")
    if kernel.startswith("tc"):
        names.add("tf32_in_place")    # a TF32 launch on the tensor cores (operands rounded by the TMA loads)
    return names


def _backend(precision):
    return "ffma" if precision == "fp32" else "tcgen05"


def _pick(native, family):
    precision, candidates = FAMILIES[family]
    for shape in candidates:
        plan = native.plan(_backend(precision), *shape, precision=precision)
        if family in _family_of(plan) and (family != "tf32_in_place" or precision == "tf32"):
            return precision, shape, plan
    pytest.fail(f"no candidate shape of {family} gets that launch plan: {candidates}")


@pytest.mark.parametrize("family", sorted(FAMILIES))
def test_progress_wait_that_runs_out_poisons_the_output_and_leaves_the_context_usable(native, family):
    precision, (m, k, n), plan = _pick(native, family)
    a_np = po.seeded_uniform((m, k), 7 * m + k)
    b_np = po.seeded_uniform((k, n), 11 * n + k)
    dtype = getattr(torch, INPUT_DTYPES[precision])
    a = torch.from_numpy(a_np).to(device="cuda", dtype=dtype)
    b = torch.from_numpy(b_np).to(device="cuda", dtype=dtype)
    out = torch.zeros((m, n), dtype=torch.float32, device="cuda")
    run = native.prepare(_backend(precision), a, b, out, precision=precision)
    assert native.device_status() == 0
    native.set_wait_limit(1)
    try:
        run()
        status = native.device_status()
    finally:
        native.set_wait_limit(0)
    assert status & (LOAD | MMA | EPILOGUE), f"{family} {plan}: status {status:#x}"
    assert not status & DRAIN, f"{family} {plan}: a drain wait ran out (status {status:#x})"
    timed_out = out.cpu().numpy()
    assert np.isnan(timed_out).any(), f"{family} {plan}: no NaN in the output of a timed-out launch"
    nan_rows = np.flatnonzero(np.isnan(timed_out).any(axis=1))[:4]
    with pytest.raises(RuntimeError):
        po.sampled_reference(a_np, b_np, precision, nan_rows).verify(timed_out[nan_rows], f"{family} timed out")

    out.fill_(float("nan"))
    run()
    torch.cuda.synchronize()
    assert torch.isfinite(out).all().item()
    rows = np.unique(np.concatenate([[0, m - 1], np.random.default_rng(m + n).integers(0, m, 8)]))
    po.sampled_reference(a_np, b_np, precision, rows).verify(
        out[torch.from_numpy(rows).cuda()].cpu().numpy(), f"{family} after the timeout, sampled rows")
    assert native.device_status() == 0


def test_wait_limit_rejects_bad_values(native):
    with pytest.raises(ValueError):
        native.set_wait_limit(-1)
    with pytest.raises(RuntimeError):
        native.set_wait_limit(3_000_000_000)
    native.set_wait_limit(0)
