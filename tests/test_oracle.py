"""The CPU oracle against the reference's own known answers (tests/golden/reference_kats.json, transcribed from
crates/staleynet-cuda/src/reference.rs:177-307 and checked there by tests/golden/make_golden.py) and against the
published SplitMix64 sequence. These pins are what make the oracle a trustworthy checker for the GPU tests."""
import json
from pathlib import Path

import numpy as np
import pytest

from oracle import oracle as o

KATS = json.loads((Path(__file__).parent / "golden" / "reference_kats.json").read_text())


def kat_product(c):
    b = c["batch"]
    return o.product(c["rows"], c["cols"], c["inner"],
                     o.storage_strides(c["left_transposed"], c["rows"], c["inner"], b["left"]),
                     o.storage_strides(c["right_transposed"], c["inner"], c["cols"], b["right"]),
                     b["output"], c["scale"], c["accumulate"])


@pytest.mark.parametrize("case", KATS["matmul"], ids=lambda c: c["name"])
def test_matmul_known_answers(case):
    out = np.array(case["initial"], np.float32)
    o.matmul(kat_product(case), case["batch"]["count"], np.array(case["left"], np.float32),
             np.array(case["right"], np.float32), out)
    assert out.tolist() == case["expected"]


@pytest.mark.parametrize("case", KATS["matmul"], ids=lambda c: c["name"])
def test_matmul_f64_agrees_on_known_answers(case):
    out = np.array(case["initial"], np.float64)
    o.matmul_f64(kat_product(case), case["batch"]["count"], np.array(case["left"], np.float32),
                 np.array(case["right"], np.float32), out)
    np.testing.assert_allclose(out, case["expected"], rtol=0, atol=1e-12)


@pytest.mark.parametrize("case", KATS["causal_softmax"], ids=lambda c: c["name"])
def test_causal_softmax_known_answers(case):
    s = np.array(case["scores"], np.float32)
    o.causal_softmax(s, case["queries"], case["keys"], case["scale"], case["query_offset"])
    np.testing.assert_allclose(s, case["expected"], atol=case["tolerance"], rtol=0)


def test_causal_softmax_applies_scale_and_offset():
    # reference.rs:282-293
    s = np.array([1.0, 2.0, 3.0, 1.0, 2.0, 3.0], np.float32)
    o.causal_softmax(s, 2, 3, 0.5, 1)
    assert abs(s[:3].sum() - 1) < 1e-6 and abs(s[3:].sum() - 1) < 1e-6
    assert s[0] < s[1] and s[2] == 0.0 and s[3] < s[4] < s[5]


@pytest.mark.parametrize("case", KATS["softmax_backward"], ids=lambda c: c["name"])
def test_softmax_backward_known_answers(case):
    g = np.array(case["grad"], np.float32)
    o.softmax_backward(np.array(case["probabilities"], np.float32), g, case["cols"])
    np.testing.assert_allclose(g, case["expected"], atol=case["tolerance"], rtol=0)
    assert abs(float(g.sum())) < 1e-6


def test_gelu_known_answers_and_derivative():
    case = KATS["gelu"][0]
    for x, want, tol in case["points"]:
        assert abs(o.gelu(np.array([x], np.float32))[0] - want) <= tol
    for x, want, tol in case["derivative_points"]:
        assert abs(o.gelu_derivative(np.array([x], np.float32))[0] - want) <= tol
    h = 1e-3
    for x in (-1.0, 0.0, 1.0):  # reference.rs:234-238
        fd = (o.gelu(np.array([x + h], np.float32))[0] - o.gelu(np.array([x - h], np.float32))[0]) / (2 * h)
        assert abs(o.gelu_derivative(np.array([x], np.float32))[0] - fd) <= 2e-3


def test_splitmix64_matches_the_published_sequence():
    k = KATS["splitmix64"]
    r = o.Random(k["seed"])
    assert [r.next_u64() for _ in k["outputs"]] == [int(v, 16) for v in k["outputs"]]


def test_random_streams_behave_like_the_reference():
    # random.rs tests: same seed repeats, different seeds diverge, uniform in [0,1), below in range, normal ~N(0,1)
    a, b = o.Random(42), o.Random(42)
    assert a.next_u64() == b.next_u64() and a.uniform() == b.uniform() and a.normal() == b.normal()
    assert o.Random(1).next_u64() != o.Random(2).next_u64()
    r = o.Random(3)
    u = [r.uniform() for _ in range(1000)]
    assert all(0.0 <= v < 1.0 for v in u) and len(set(u)) > 1
    r = o.Random(4)
    assert all(r.below(10) < 10 for _ in range(1000))
    x = o.Random(6).normals(20000)
    assert abs(float(x.mean())) < 0.05 and abs(float(x.var()) - 1.0) < 0.05


def test_normals_fill_equals_repeated_normal():
    a, b = o.Random(0), o.Random(0)
    filled = a.normals(64, std=0.5)
    single = np.array([b.normal() * np.float32(0.5) for _ in range(64)], np.float32)
    assert np.array_equal(filled, single)


def test_lcg_values_are_deterministic_and_in_range():
    v = o.lcg_values(4096, 1)
    assert np.array_equal(v, o.lcg_values(4096, 1))
    assert float(v.min()) >= -1.0 and float(v.max()) < 1.0
    assert not np.array_equal(v, o.lcg_values(4096, 2))


def test_tf32_rounding_is_round_to_nearest_ties_away():
    x = np.array([1.0, 1.0 + 2.0**-11, 1.0 + 2.0**-12, -(1.0 + 2.0**-11), 1.0 + 3 * 2.0**-11, np.inf], np.float32)
    r = o.round_tf32(x)
    assert r[0] == 1.0
    assert r[1] == 1.0 + 2.0**-10  # exactly half an ulp: away from zero
    assert r[2] == 1.0
    assert r[3] == -(1.0 + 2.0**-10)
    assert r[4] == 1.0 + 2 * 2.0**-10
    assert np.isinf(r[5])
    bits = r[:5].view(np.uint32)
    assert np.all(bits & 0x1FFF == 0)


def test_bf16_rounding_is_round_to_nearest_even():
    x = np.array([1.0, 1.0 + 2.0**-8, 1.0 + 3 * 2.0**-8, 1.0 + 2.0**-9, -2.5], np.float32)
    r, bits = o.round_bf16(x)
    assert r[0] == 1.0
    assert r[1] == 1.0  # tie to even
    assert r[2] == 1.0 + 4 * 2.0**-8  # tie to even (upwards)
    assert r[3] == 1.0
    assert r[4] == -2.5
    assert np.array_equal(bits, (r.view(np.uint32) >> 16).astype(np.uint16))


@pytest.mark.parametrize("lt,rt", [(False, False), (True, False), (False, True), (True, True)])
def test_parallel_rows_match_serial_bit_for_bit(lt, rt):
    rows, cols, inner, count = 37, 29, 53, 2
    left = o.lcg_values(count * rows * inner, 1)
    right = o.lcg_values(count * inner * cols, 2)
    init = o.lcg_values(count * rows * cols, 3)
    p = o.product(rows, cols, inner, o.storage_strides(lt, rows, inner, rows * inner),
                  o.storage_strides(rt, inner, cols, inner * cols), rows * cols, 0.7, True)
    a, b = init.copy(), init.copy()
    o.matmul(p, count, left, right, a)
    o.matmul_rows(p, count, left, right, b, 0, rows, 4)
    assert np.array_equal(a, b)


def test_f32_oracle_is_close_to_f64_on_random_data():
    rows, cols, inner = 64, 48, 700
    left = o.lcg_values(rows * inner, 1)
    right = o.lcg_values(inner * cols, 2)
    p = o.product(rows, cols, inner, (inner, 1, 0), (cols, 1, 0), 0)
    f32 = np.zeros(rows * cols, np.float32)
    f64 = np.zeros(rows * cols, np.float64)
    o.matmul(p, 1, left, right, f32)
    o.matmul_f64(p, 1, left, right, f64)
    assert o.relative_error(f64, f32) < 1e-5


def _check_entry(value, expected):
    if expected is None:
        return
    if expected == "positive":
        assert value > 0.0
    elif expected == "negative":
        assert value < 0.0
    elif expected == "finite":
        assert np.isfinite(value)
    else:
        want, tol = expected
        assert abs(value - want) <= tol, (value, want)


@pytest.mark.parametrize("case", KATS["cross_entropy"], ids=lambda c: c["name"])
def test_cross_entropy_matches_the_reference_known_answers(case):
    """reference.rs:309-366 through the oracle's restatement of reference::cross_entropy."""
    logits = np.array(case["logits"], dtype=np.float32)
    targets = np.array(case["targets"], dtype=np.uint32)
    h = case["head"]
    rows = len(case["expected_losses"])
    losses = np.full(rows, 9.0, dtype=np.float32)
    grad = np.full(logits.size, 7.0, dtype=np.float32)
    o.cross_entropy(logits, targets, case["cols"], h["column_offset"], h["classes"], h["target_stride"],
                    h["target_offset"], h["grad_scale"], losses, grad)
    for value, expected in zip(losses, case["expected_losses"]):
        _check_entry(float(value), expected)
    for value, expected in zip(grad, case["expected_grad"]):
        _check_entry(float(value), expected)


@pytest.mark.parametrize("case", KATS["rms_norm"], ids=lambda c: c["name"])
def test_rms_norm_matches_the_reference_known_answers(case):
    """reference.rs:247-265 through the oracle's restatement of rms_norm_forward / rms_norm_backward."""
    if "output_grad" in case:
        dx, dg = o.rms_norm_backward(np.array(case["output_grad"]), np.array(case["input"]), np.array(case["gain"]),
                                     np.array(case["inv_rms"]), case["cols"])
        for value, expected in zip(dx, case["expected_input_grad"]):
            _check_entry(float(value), expected)
        for value, expected in zip(dg, case["expected_gain_grad"]):
            _check_entry(float(value), expected)
    else:
        out, inv = o.rms_norm_forward(np.array(case["input"]), np.array(case["gain"]), case["cols"], case["epsilon"])
        for value, expected in zip(inv, case["expected_inv_rms"]):
            _check_entry(float(value), expected)
        for value, expected in zip(out, case["expected_output"]):
            _check_entry(float(value), expected)


def test_adamw_matches_the_reference_parity_formula():
    """The update formula of kernels_match_reference.rs:299-327 (written out there in f32) against the oracle."""
    c = KATS["adamw"]
    w = o.lcg_values(c["count"], c["parameter_seed"])
    g = o.lcg_values(c["count"], c["gradient_seed"])
    f32 = np.float32
    b1, b2, lr, eps, wd = f32(c["beta1"]), f32(c["beta2"]), f32(c["learning_rate"]), f32(c["epsilon"]), f32(c["weight_decay"])
    mean = b1 * f32(c["initial_mean"]) + (f32(1) - b1) * g
    var = b2 * f32(c["initial_variance"]) + (f32(1) - b2) * g * g
    mean_hat = mean / (f32(1) - b1 ** 2)
    var_hat = var / (f32(1) - b2 ** 2)
    expected = w - lr * (mean_hat / (np.sqrt(var_hat) + eps) + wd * w)
    p = w.copy()
    m = np.full(c["count"], c["initial_mean"], np.float32)
    v = np.full(c["count"], c["initial_variance"], np.float32)
    o.adamw_step(p, g, m, v, c["learning_rate"], c["beta1"], c["beta2"], c["epsilon"], c["weight_decay"], c["step"])
    assert o.relative_error(expected, p) < 1e-5


def test_head_permutes_follow_the_reference_formula():
    # The layout of the reference's split_and_merge_heads_follow_the_layout_formula
    # (crates/staleynet-cuda/tests/kernels_match_reference.rs:199-231): dense(2, 5, 3, 4, 3*12 + 2, 13).in_cache(9, 2),
    # inputs random_values(n, 12); every moved element lands at its formula index and a merge restores exactly the
    # head columns, zero elsewhere.
    from staleynet_b200._ffi import HeadLayout

    L = HeadLayout.dense(2, 5, 3, 4, 3 * 12 + 2, 13).in_cache(9, 2)
    packed = o.lcg_values(L.batch * L.time * L.width, 12)
    head_major = np.zeros(L.batch * L.heads * L.time_capacity * L.head_dim, np.float32)
    o.split_heads(packed, head_major, L)
    for b in range(L.batch):
        for h in range(L.heads):
            for t in range(L.time):
                for d in range(L.head_dim):
                    src = (b * L.time + t) * L.width + L.column_offset + h * L.head_dim + d
                    dst = ((b * L.heads + h) * L.time_capacity + L.time_offset + t) * L.head_dim + d
                    assert head_major[dst] == packed[src]
    merged = np.zeros_like(packed)
    o.merge_heads(head_major, merged, L)
    cols = np.arange(packed.size) % L.width
    inside = (cols >= L.column_offset) & (cols < L.column_offset + L.heads * L.head_dim)
    assert np.array_equal(merged, np.where(inside, packed, 0.0).astype(np.float32))
