"""Writes tests/golden/reference_kats.json: the known-answer vectors of the reference's own tests for the GEMM
path and its neighbours, each with the file:line it comes from.

    python tests/golden/make_golden.py [--reference /path/to/staleynet]

The vectors are transcribed below; when the reference checkout is given (by --reference or the STALEYNET_REFERENCE
environment variable), every literal is checked to occur verbatim at the cited lines before the fixture is written,
so the fixture cannot drift from the reference's tests. The GPU box never runs this script; tests read only the JSON.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
DEFAULT_REFERENCE = Path(os.environ["STALEYNET_REFERENCE"]) if os.environ.get("STALEYNET_REFERENCE") else None
REF_FILE = "crates/staleynet-cuda/src/reference.rs"

# (name, source lines, literal snippets that must appear in those lines, case data)
MATMUL_KATS = [
    {
        "name": "matmul_overwrites_a_row_major_product",
        "source": f"{REF_FILE}:177-187",
        "snippets": ["MatmulSpec::new(2, 3, 2)", "[1.0, 2.0, 3.0, 4.0]", "[5.0, 6.0, 7.0, 8.0, 9.0, 10.0]",
                     "[21.0, 24.0, 27.0, 47.0, 54.0, 61.0]"],
        "rows": 2, "cols": 3, "inner": 2, "left_transposed": False, "right_transposed": False,
        "batch": {"count": 1, "left": 0, "right": 0, "output": 0}, "scale": 1.0, "accumulate": False,
        "left": [1.0, 2.0, 3.0, 4.0], "right": [5.0, 6.0, 7.0, 8.0, 9.0, 10.0], "initial": [0.0] * 6,
        "expected": [21.0, 24.0, 27.0, 47.0, 54.0, 61.0],
    },
    {
        "name": "matmul_scales_and_accumulates_into_the_existing_output",
        "source": f"{REF_FILE}:189-199",
        "snippets": ["MatmulSpec::new(2, 3, 2).scaled(0.5).accumulate()", "[1.0f32; 6]",
                     "[11.5, 13.0, 14.5, 24.5, 28.0, 31.5]"],
        "rows": 2, "cols": 3, "inner": 2, "left_transposed": False, "right_transposed": False,
        "batch": {"count": 1, "left": 0, "right": 0, "output": 0}, "scale": 0.5, "accumulate": True,
        "left": [1.0, 2.0, 3.0, 4.0], "right": [5.0, 6.0, 7.0, 8.0, 9.0, 10.0], "initial": [1.0] * 6,
        "expected": [11.5, 13.0, 14.5, 24.5, 28.0, 31.5],
    },
    {
        "name": "matmul_honours_transposed_storage",
        "source": f"{REF_FILE}:201-211",
        "snippets": ["MatmulSpec::new(2, 2, 2).left_transposed()", "[5.0, 6.0, 7.0, 8.0]",
                     "[26.0, 30.0, 38.0, 44.0]"],
        "rows": 2, "cols": 2, "inner": 2, "left_transposed": True, "right_transposed": False,
        "batch": {"count": 1, "left": 0, "right": 0, "output": 0}, "scale": 1.0, "accumulate": False,
        "left": [1.0, 2.0, 3.0, 4.0], "right": [5.0, 6.0, 7.0, 8.0], "initial": [0.0] * 4,
        "expected": [26.0, 30.0, 38.0, 44.0],
    },
    {
        "name": "matmul_broadcasts_batched_operands",
        "source": f"{REF_FILE}:213-224",
        "snippets": ["BatchStrides { count: 2, left: 4, right: 0, output: 4 }",
                     "[1.0, 2.0, 3.0, 4.0, 5.0, 6.0, 7.0, 8.0]", "[1.0, 0.0, 0.0, 1.0]",
                     "assert_eq!(output, left)"],
        "rows": 2, "cols": 2, "inner": 2, "left_transposed": False, "right_transposed": False,
        "batch": {"count": 2, "left": 4, "right": 0, "output": 4}, "scale": 1.0, "accumulate": False,
        "left": [1.0, 2.0, 3.0, 4.0, 5.0, 6.0, 7.0, 8.0], "right": [1.0, 0.0, 0.0, 1.0], "initial": [0.0] * 8,
        "expected": [1.0, 2.0, 3.0, 4.0, 5.0, 6.0, 7.0, 8.0],
    },
]

SOFTMAX_KATS = [
    {
        "name": "causal_softmax_masks_future_keys",
        "source": f"{REF_FILE}:267-280",
        "snippets": ["[1.0, 100.0, 100.0, 1.0, 2.0, 100.0]", "causal_softmax(&mut scores, 2, 3, 1.0, 0)",
                     "0.268_941_4", "0.731_058_6"],
        "scores": [1.0, 100.0, 100.0, 1.0, 2.0, 100.0], "queries": 2, "keys": 3, "scale": 1.0, "query_offset": 0,
        "expected": [1.0, 0.0, 0.0, 0.2689414, 0.7310586, 0.0], "tolerance": 1e-6,
    },
]

SOFTMAX_BACKWARD_KATS = [
    {
        "name": "softmax_backward_projects_out_the_weighted_sum",
        "source": f"{REF_FILE}:295-306",
        "snippets": ["[0.25, 0.25, 0.5]", "[1.0, 2.0, 3.0]", "-0.3125", "-0.0625", "0.375"],
        "probabilities": [0.25, 0.25, 0.5], "grad": [1.0, 2.0, 3.0], "cols": 3,
        "expected": [-0.3125, -0.0625, 0.375], "tolerance": 1e-6,
    },
]

GELU_KATS = [
    {
        "name": "gelu_matches_known_values_and_its_finite_difference_derivative",
        "source": f"{REF_FILE}:226-239",
        "snippets": ["close(gelu(0.0), 0.0, 1e-6)", "close(gelu(1.0), 0.841_191, 1e-4)",
                     "close(gelu_derivative(0.0), 0.5, 1e-6)"],
        "points": [[0.0, 0.0, 1e-6], [1.0, 0.841191, 1e-4]],
        "derivative_points": [[0.0, 0.5, 1e-6]],
    },
]

# Cross-entropy of one head (reference::cross_entropy, reference.rs:139-166). EMPTY_TOKEN is u32::MAX
# (crates/staleynet-cuda/src/kernels/mod.rs:46); 7.0 marks gradient entries the head must leave untouched.
EMPTY = 0xFFFFFFFF
CROSS_ENTROPY_KATS = [
    {
        "name": "cross_entropy_writes_losses_and_gradients_for_the_target_head",
        "source": f"{REF_FILE}:309-330",
        "snippets": ["[1.0, 2.0, 3.0, 0.0, 0.0, 0.0, 0.0, 0.0]", "[2u32, 0]",
                     "column_offset: 0, classes: 3, target_stride: 1, target_offset: 0, grad_scale: 1.0",
                     "0.407_606", "1.098_612", "0.090_03", "0.244_73", "-0.334_76", "-0.666_667", "0.333_333"],
        "logits": [1.0, 2.0, 3.0, 0.0, 0.0, 0.0, 0.0, 0.0], "targets": [2, 0], "cols": 4,
        "head": {"column_offset": 0, "classes": 3, "target_stride": 1, "target_offset": 0, "grad_scale": 1.0},
        "expected_losses": [[0.407606, 1e-5], [1.098612, 1e-5]],
        "expected_grad": [[0.09003, 1e-4], [0.24473, 1e-4], [-0.33476, 1e-4], [7.0, 0.0],
                          [-0.666667, 1e-5], [0.333333, 1e-5], [0.333333, 1e-5], [7.0, 0.0]],
    },
    {
        "name": "cross_entropy_skips_empty_targets",
        "source": f"{REF_FILE}:333-347",
        "snippets": ["[EMPTY_TOKEN, 0]", "assert_eq!(losses[0], 0.0)", "assert_eq!(&grad[0..3], &[0.0, 0.0, 0.0])",
                     "assert_eq!(grad[3], 7.0)", "assert!(grad[4] < 0.0 && grad[5] > 0.0 && grad[6] > 0.0)"],
        "logits": [1.0, 2.0, 3.0, 0.0, 0.0, 0.0, 0.0, 0.0], "targets": [EMPTY, 0], "cols": 4,
        "head": {"column_offset": 0, "classes": 3, "target_stride": 1, "target_offset": 0, "grad_scale": 1.0},
        "expected_losses": [[0.0, 0.0], None],
        "expected_grad": [[0.0, 0.0], [0.0, 0.0], [0.0, 0.0], [7.0, 0.0], "negative", "positive", "positive", [7.0, 0.0]],
    },
    {
        "name": "cross_entropy_honours_head_offsets_and_gradient_scale",
        "source": f"{REF_FILE}:350-366",
        "snippets": ["[1.0, 2.0, 3.0, 4.0, 5.0, 1.0, 2.0, 3.0, 4.0, 5.0]", "[0u32, 1, 0, 0]",
                     "column_offset: 2, classes: 2, target_stride: 2, target_offset: 1, grad_scale: 0.5",
                     "assert_eq!(&grad[0..2], &[7.0, 7.0])", "assert_eq!(grad[4], 7.0)", "assert_eq!(grad[9], 7.0)"],
        "logits": [1.0, 2.0, 3.0, 4.0, 5.0, 1.0, 2.0, 3.0, 4.0, 5.0], "targets": [0, 1, 0, 0], "cols": 5,
        "head": {"column_offset": 2, "classes": 2, "target_stride": 2, "target_offset": 1, "grad_scale": 0.5},
        "expected_losses": ["positive", "positive"],
        "expected_grad": [[7.0, 0.0], [7.0, 0.0], "finite", "finite", [7.0, 0.0], [7.0, 0.0], [7.0, 0.0], "finite",
                          "finite", [7.0, 0.0]],
    },
]

RMS_NORM_KATS = [
    {
        "name": "rms_norm_forward_matches_the_definition",
        "source": f"{REF_FILE}:247-254",
        "snippets": ["rms_norm_forward(&[3.0, 4.0], &[1.0, 1.0], 2, 0.0)", "0.282_842_7", "0.848_528_1",
                     "1.131_370_8"],
        "input": [3.0, 4.0], "gain": [1.0, 1.0], "cols": 2, "epsilon": 0.0,
        "expected_inv_rms": [[0.2828427, 1e-6]], "expected_output": [[0.8485281, 1e-6], [1.1313708, 1e-6]],
    },
    {
        "name": "rms_norm_backward_matches_the_hand_derived_gradient",
        "source": f"{REF_FILE}:256-265",
        "snippets": ["[0.282_842_7f32]", "rms_norm_backward(&[1.0, 0.0], &[3.0, 4.0], &[1.0, 1.0], &inv_rms, 2)",
                     "0.181_0", "-0.135_8", "0.848_528_1"],
        "output_grad": [1.0, 0.0], "input": [3.0, 4.0], "gain": [1.0, 1.0], "inv_rms": [0.2828427], "cols": 2,
        "expected_input_grad": [[0.181, 1e-3], [-0.1358, 1e-3]], "expected_gain_grad": [[0.8485281, 1e-6], [0.0, 1e-6]],
    },
]

# The AdamW parity test's settings (tests/kernels_match_reference.rs:299-327; its expected values are computed by
# the formula there, which the oracle restates).
ADAMW_CASE = {
    "source": "crates/staleynet-cuda/tests/kernels_match_reference.rs:299-327",
    "snippets": ["learning_rate: 1e-3, beta1: 0.9, beta2: 0.95, epsilon: 1e-8, weight_decay: 0.1, step: 2",
                 "(initial_mean, initial_variance) = (0.01f32, 0.02f32)", "random_values(shape.len(), 16)",
                 "random_values(shape.len(), 17)", "Shape::vector(300)"],
    "count": 300, "parameter_seed": 16, "gradient_seed": 17, "learning_rate": 1e-3, "beta1": 0.9, "beta2": 0.95,
    "epsilon": 1e-8, "weight_decay": 0.1, "step": 2, "initial_mean": 0.01, "initial_variance": 0.02,
}

# SplitMix64 is the reference's generator (crates/staleynet-model/src/random.rs:4-46). Its published output for
# state 0 (Vigna's splitmix64.c, the algorithm of Steele, Lea & Flood 2014) pins next_u64.
SPLITMIX_KATS = {
    "source": "crates/staleynet-model/src/random.rs:4-46",
    "seed": 0,
    "outputs": ["0xe220a8397b1dcdaf", "0x6e789e6aa1b965f4", "0x06c45d188009454f"],
}


def check_against_reference(reference: Path) -> None:
    lines = (reference / REF_FILE).read_text().splitlines()
    for case in MATMUL_KATS + SOFTMAX_KATS + SOFTMAX_BACKWARD_KATS + GELU_KATS + CROSS_ENTROPY_KATS:
        span = case["source"].rsplit(":", 1)[1]
        lo, hi = (int(x) for x in span.split("-"))
        text = "\n".join(lines[lo - 1:hi])
        for snippet in case["snippets"]:
            if snippet not in text:
                raise SystemExit(f"{case['name']}: {snippet!r} not found at {case['source']}")
    for case in RMS_NORM_KATS:
        span = case["source"].rsplit(":", 1)[1]
        lo, hi = (int(x) for x in span.split("-"))
        text = "\n".join(lines[lo - 1:hi])
        for snippet in case["snippets"]:
            if snippet not in text:
                raise SystemExit(f"{case['name']}: {snippet!r} not found at {case['source']}")
    test_lines = (reference / "crates/staleynet-cuda/tests/kernels_match_reference.rs").read_text().splitlines()
    text = "\n".join(test_lines[298:327])
    for snippet in ADAMW_CASE["snippets"]:
        if snippet not in text:
            raise SystemExit(f"adamw: {snippet!r} not found at {ADAMW_CASE['source']}")
    random_src = (reference / "crates/staleynet-model/src/random.rs").read_text()
    for constant in ("0x9E37_79B9_7F4A_7C15", "0xBF58_476D_1CE4_E5B9", "0x94D0_49BB_1331_11EB"):
        if constant not in random_src:
            raise SystemExit(f"SplitMix64 constant {constant} not found in random.rs")


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", type=Path, default=DEFAULT_REFERENCE)
    args = ap.parse_args(argv)
    checked = False
    if args.reference is not None and (args.reference / REF_FILE).exists():
        check_against_reference(args.reference)
        checked = True
    out = {
        "generated_by": "tests/golden/make_golden.py",
        "checked_against_reference_source": checked,
        "matmul": [{k: v for k, v in c.items() if k != "snippets"} for c in MATMUL_KATS],
        "causal_softmax": [{k: v for k, v in c.items() if k != "snippets"} for c in SOFTMAX_KATS],
        "softmax_backward": [{k: v for k, v in c.items() if k != "snippets"} for c in SOFTMAX_BACKWARD_KATS],
        "gelu": [{k: v for k, v in c.items() if k != "snippets"} for c in GELU_KATS],
        "cross_entropy": [{k: v for k, v in c.items() if k != "snippets"} for c in CROSS_ENTROPY_KATS],
        "rms_norm": [{k: v for k, v in c.items() if k != "snippets"} for c in RMS_NORM_KATS],
        "adamw": {k: v for k, v in ADAMW_CASE.items() if k != "snippets"},
        "splitmix64": SPLITMIX_KATS,
    }
    (HERE / "reference_kats.json").write_text(json.dumps(out, indent=1) + "\n")
    print(f"wrote {HERE / 'reference_kats.json'} (checked against reference source: {checked})")
    return 0


if __name__ == "__main__":
    sys.exit(main())
