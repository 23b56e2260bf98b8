"""Softmax cross-entropy on the GPU (snb_cross_entropy, snb_head_cross_entropy) against the oracle's restatement of
reference::cross_entropy (reference.rs:139-166), mirroring the reference's own parity test
(crates/staleynet-cuda/tests/kernels_match_reference.rs:277-297) and known answers (reference.rs:309-366)."""
import json
from pathlib import Path

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import oracle as o  # noqa: E402
from staleynet_b200 import _ffi  # noqa: E402
from staleynet_b200.matmul import EMPTY_TOKEN, CrossEntropyHead, Gpu, MatmulSpec  # noqa: E402

pytestmark = pytest.mark.gpu

KATS = json.loads((Path(__file__).parent / "golden" / "reference_kats.json").read_text())["cross_entropy"]


def _targets_tensor(values):
    return torch.from_numpy(np.asarray(values, dtype=np.uint32).view(np.int32)).cuda()


def test_cross_entropy_matches_the_reference_parity_case():
    """kernels_match_reference.rs:277-297: 13x50 logits, head at column 10 with 37 classes, 2 targets per row (the
    second one used), every 7th target empty, gradient scale 0.25; max|d|/max|ref| < 1e-5."""
    rows, cols = 13, 50
    head = CrossEntropyHead(column_offset=10, classes=37, target_stride=2, target_offset=1, grad_scale=0.25)
    logits = o.lcg_values(rows * cols, 15)
    targets = np.array([EMPTY_TOKEN if i % 7 == 0 else (i * 5 % head.classes) for i in range(rows * 2)],
                       dtype=np.uint32)
    e_losses = np.zeros(rows, np.float32)
    e_grad = np.zeros(rows * cols, np.float32)
    o.cross_entropy(logits, targets, cols, head.column_offset, head.classes, head.target_stride, head.target_offset,
                    head.grad_scale, e_losses, e_grad)
    gpu = Gpu(0)
    losses = torch.zeros(rows, device="cuda")
    grad = torch.zeros(rows, cols, device="cuda")
    gpu.cross_entropy(torch.from_numpy(logits).cuda().view(rows, cols), _targets_tensor(targets), head, losses, grad)
    torch.cuda.synchronize()
    assert o.relative_error(e_losses, losses.cpu().numpy()) < 1e-5
    assert o.relative_error(e_grad, grad.cpu().numpy().ravel()) < 1e-5


@pytest.mark.parametrize("case", KATS, ids=lambda c: c["name"])
def test_cross_entropy_known_answers_on_the_gpu(case):
    from test_oracle import _check_entry

    h = case["head"]
    logits = np.array(case["logits"], dtype=np.float32)
    rows = len(case["expected_losses"])
    cols = case["cols"]
    gpu = Gpu(0)
    losses = torch.full((rows,), 9.0, device="cuda")
    grad = torch.full((rows, cols), 7.0, device="cuda")
    gpu.cross_entropy(torch.from_numpy(logits).cuda().view(rows, cols), _targets_tensor(case["targets"]),
                      CrossEntropyHead(**h), losses, grad)
    torch.cuda.synchronize()
    for value, expected in zip(losses.cpu().numpy(), case["expected_losses"]):
        _check_entry(float(value), expected)
    for value, expected in zip(grad.cpu().numpy().ravel(), case["expected_grad"]):
        _check_entry(float(value), expected)


def test_cross_entropy_checks_in_the_reference_order():
    gpu = Gpu(0)
    logits = torch.zeros(4, 8, device="cuda")
    grad = torch.zeros(4, 8, device="cuda")
    losses = torch.zeros(4, device="cuda")
    targets = _targets_tensor([0] * 8)
    with pytest.raises(AssertionError, match="head exceeds logits"):
        gpu.cross_entropy(logits, targets, CrossEntropyHead(4, 5, 2, 0, 1.0), losses, grad)
    with pytest.raises(AssertionError, match="losses too small"):
        gpu.cross_entropy(logits, targets, CrossEntropyHead(0, 8, 2, 0, 1.0), losses[:3], grad)
    with pytest.raises(AssertionError, match="too few targets"):
        gpu.cross_entropy(logits, targets, CrossEntropyHead(0, 8, 3, 0, 1.0), losses, grad)


def test_cross_entropy_codebook_heads_take_the_register_path():
    """16 heads of 1024 classes (BASELINE's codebooks), ragged rows: each head through snb_cross_entropy."""
    rows, books, size = 300, 16, 1024
    rng = np.random.default_rng(3)
    logits = (rng.standard_normal(rows * books * size) * 3).astype(np.float32)
    targets = rng.integers(0, size, rows * books).astype(np.uint32)
    targets[::11] = EMPTY_TOKEN
    gpu = Gpu(0)
    lg = torch.from_numpy(logits).cuda().view(rows, books * size)
    tg = _targets_tensor(targets)
    grad = torch.zeros_like(lg)
    for c in range(books):
        head = CrossEntropyHead(c * size, size, books, c, 1.0 / (rows * books))
        losses = torch.zeros(rows, device="cuda")
        gpu.cross_entropy(lg, tg, head, losses, grad)
        e_losses = np.zeros(rows, np.float32)
        e_grad = np.zeros(rows * books * size, np.float32)
        o.cross_entropy(logits, targets, books * size, c * size, size, books, c, head.grad_scale, e_losses, e_grad)
        torch.cuda.synchronize()
        assert o.relative_error(e_losses, losses.cpu().numpy()) < 1e-5
        got = grad.cpu().numpy().reshape(rows, books, size)[:, c]
        assert o.relative_error(e_grad.reshape(rows, books, size)[:, c], got) < 1e-5


@pytest.mark.parametrize("logit_type", ["bf16-in-place", "f32"])
def test_head_cross_entropy_matches_the_oracle_composition(logit_type):
    """The output layer (x W + b, then every codebook's cross-entropy) in one call, against the oracle on the same
    bf16 operands: loss sums per codebook and the gradient (relative Frobenius <= 1e-2 with bf16 logits, whose
    rounding the gradient inherits; 1e-4 with f32 logits)."""
    rows, width, books, size = 300, 768, 16, 1024
    cols = books * size
    g = torch.Generator(device="cuda")
    g.manual_seed(11)
    x = torch.randn(rows, width, device="cuda", generator=g).bfloat16()
    w = (torch.randn(width, cols, device="cuda", generator=g) / width ** 0.5).bfloat16()
    bias = torch.randn(cols, device="cuda", generator=g) * 0.1
    rng = np.random.default_rng(5)
    targets = rng.integers(0, size, rows * books).astype(np.uint32)
    targets[::13] = EMPTY_TOKEN
    valid = (targets.reshape(rows, books) != EMPTY_TOKEN).sum(axis=0)
    scales = torch.tensor([1.0 / (v * books) for v in valid], dtype=torch.float32, device="cuda")
    gpu = Gpu(0)
    loss_sums = torch.full((books,), 5.0, device="cuda")
    if logit_type == "f32":
        logits = torch.empty(rows, cols, device="cuda")
        grad = torch.empty(rows, cols, device="cuda")
    else:
        logits = torch.empty(rows, cols, device="cuda", dtype=torch.bfloat16)
        grad = logits
    gpu.head_cross_entropy(MatmulSpec.new(rows, cols, width), x, w, logits, _targets_tensor(targets), books, scales,
                           loss_sums, grad, bias=bias)
    torch.cuda.synchronize()
    assert _ffi.load().snb_device_status() == _ffi.OK
    z = (x.double() @ w.double() + bias.double()).float().cpu().numpy().ravel()
    e_grad = np.zeros(rows * cols, np.float32)
    tol = 1e-4 if logit_type == "f32" else 1e-2
    got = grad.float().cpu().numpy().reshape(rows, books, size)
    for c in range(books):
        e_losses = np.zeros(rows, np.float32)
        o.cross_entropy(z, targets, cols, c * size, size, books, c, float(scales[c]), e_losses, e_grad)
        assert abs(float(loss_sums[c]) - float(e_losses.sum())) <= 2e-3 * abs(float(e_losses.sum())), c
        assert o.relative_frobenius(e_grad.reshape(rows, books, size)[:, c], got[:, c]) < tol, c
