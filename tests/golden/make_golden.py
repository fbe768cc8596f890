"""Generate the golden vectors that pin the CPU oracle to the reference.

Run where a checkout of the reference is available::

    python tests/golden/make_golden.py --reference /path/to/matrix-multiplication

It imports the reference's own ``src/precision.py`` (quantize_inputs,
reference_product, GemmReference) and writes ``precision_golden.npz`` beside
this script.  The tests load only the ``.npz``; nothing at test time reads the
reference checkout.
"""

from __future__ import annotations

import argparse
import importlib.util
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent

# Small shapes verified in full (reference tests/test_matmul.py:31 plus the
# smallest ragged shape of the benchmark configuration).
FULL_SHAPES = ((1, 1, 1), (7, 13, 11), (35, 37, 67), (2, 2049, 3), (31, 33, 65))
# Larger ragged shapes: only checksums and sampled entries are stored.
SUMMARY_SHAPES = ((511, 257, 129), (513, 129, 577))
PRECISIONS = ("fp32", "tf32", "fp16", "bf16")


def load_reference(root: Path):
    path = root / "src" / "precision.py"
    spec = importlib.util.spec_from_file_location("reference_precision", path)
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    return module


def quantize_probe() -> np.ndarray:
    """Inputs that exercise every rounding branch of the three formats."""
    values = []
    for fraction_bits in (10, 7):            # TF32 and BF16 ties (test_precision.py:12-19)
        step = 2.0 ** -fraction_bits
        values += [1 + step / 2, 1 + 3 * step / 2, -1 - step / 2, -1 - 3 * step / 2,
                   1 + step / 2 + 2.0 ** -23, 1 + step / 2 - 2.0 ** -23]
    step = 2.0 ** -10                        # FP16 ties and subnormals
    values += [1 + step / 2, 1 + 3 * step / 2, -1 - step / 2, 2.0 ** -24, 2.0 ** -25,
               -2.0 ** -25, 3 * 2.0 ** -26, 65504.0, 65519.0, 65520.0, 1e6]
    values += [0.0, -0.0, np.inf, -np.inf, 3.4e38, -3.4e38, 1.17549435e-38, 1e-45]
    tie_bits = np.array([0x3f801000, 0x3f803000, 0x3f800fff, 0x3f801001,
                         0xbf801000, 0xbf803000, 0xbf800fff, 0xbf801001], dtype=np.uint32)
    probe = np.concatenate([np.array(values, dtype=np.float32), tie_bits.view(np.float32),
                            np.random.default_rng(77).standard_normal(256).astype(np.float32),
                            (np.random.default_rng(78).standard_normal(64) * 1e-6).astype(np.float32)])
    return probe


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--reference", type=Path, required=True,
                        help="checkout of chudinovAI/matrix-multiplication (its src/precision.py is imported)")
    args = parser.parse_args()
    ref = load_reference(args.reference)
    out = {}
    probe = quantize_probe()
    out["probe"] = probe
    with np.errstate(over="ignore", invalid="ignore"):
        for precision in PRECISIONS:
            out[f"quantize_{precision}"] = ref.quantize_inputs(probe, precision)
        out["quantize_tf32_away"] = ref.quantize_inputs(probe, "tf32", tf32_ties="away")
    for m, k, n in FULL_SHAPES:
        seed = 1000 * m + 10 * k + n
        a = np.random.default_rng(seed).uniform(-1, 1, (m, k)).astype(np.float32)
        b = np.random.default_rng(seed + 1).uniform(-1, 1, (k, n)).astype(np.float32)
        tag = f"{m}x{k}x{n}"
        out[f"a_{tag}"] = a
        out[f"b_{tag}"] = b
        for precision in PRECISIONS:
            reference = ref.GemmReference(a, b, precision)
            out[f"rounded_{tag}_{precision}"] = reference.rounded
            out[f"bound_{tag}_{precision}"] = reference._roundoff_bound
            # verify() on the FP32 rounding of the exact product: its report is pinned too.
            report = reference.verify(reference.rounded.astype(np.float32), tag)
            out[f"ratio_{tag}_{precision}"] = np.float64(report["max_tolerance_ratio"])
    for m, k, n in SUMMARY_SHAPES:
        seed = 1000 * m + 10 * k + n
        a = np.random.default_rng(seed).uniform(-1, 1, (m, k)).astype(np.float32)
        b = np.random.default_rng(seed + 1).uniform(-1, 1, (k, n)).astype(np.float32)
        tag = f"{m}x{k}x{n}"
        for precision in PRECISIONS:
            reference = ref.GemmReference(a, b, precision)
            rows = np.arange(0, m, 37)
            out[f"sample_rows_{tag}"] = rows
            out[f"sample_{tag}_{precision}"] = reference.rounded[rows]
            out[f"checksum_{tag}_{precision}"] = np.array(
                [reference.rounded.sum(), np.abs(reference.rounded).sum(),
                 reference._roundoff_bound.max(), reference._roundoff_bound.sum()])
    np.savez_compressed(HERE / "precision_golden.npz", **out)
    print(f"wrote {HERE / 'precision_golden.npz'} ({len(out)} arrays)")


if __name__ == "__main__":
    sys.exit(main())
