"""The benchmark's training step (staleynet_b200/step.py) on a small decoder: gradient accumulation over
micro-batches (the reference's `accumulate` dW products, crates/staleynet-model/src/layers/linear.rs:55-57) gives
the sum of the micro-batches' gradients, and the loss between the passes is the codebooks' cross-entropy of the
logits (crates/staleynet-model/src/training.rs:209-235) checked against the oracle."""
import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import oracle as o  # noqa: E402
from staleynet_b200 import _ffi  # noqa: E402
from staleynet_b200.step import ModelShape, TrainingStepGemms  # noqa: E402

pytestmark = pytest.mark.gpu

SHAPE = ModelShape(blocks=2, width=256, ffn=1024, codebooks=2, codebook_size=256, tokens=1024)


def _grads(step):
    return [step.head_grad.clone()] + [f.clone() for f in step.block_grad_flat]


def _rel(a, b):
    return (torch.linalg.vector_norm((a - b).double()) / torch.linalg.vector_norm(b.double())).item()


def test_micro_batches_accumulate_into_the_sum_of_their_gradients():
    dev = torch.device("cuda", 0)
    h = torch.cuda.current_stream().cuda_stream
    scale = 1.0 / (2 * SHAPE.tokens * SHAPE.codebooks)
    both = TrainingStepGemms(SHAPE, dev, micro_batches=2, first_micro_batch=0, grad_scale=scale)
    both.run_step(h)
    g2 = _grads(both)
    parts = []
    for first in (0, 1):
        one = TrainingStepGemms(SHAPE, dev, micro_batches=1, first_micro_batch=first, grad_scale=scale)
        one.run_step(h)
        parts.append(_grads(one))
        assert torch.equal(one.inputs[0], both.inputs[first]), "micro-batch inputs come from the global stream"
    torch.cuda.synchronize()
    for acc, a, b in zip(g2, *parts):
        assert _rel(acc, a + b) < 1e-5
    assert torch.isfinite(both.loss_sums).all()


def test_step_loss_is_the_codebook_cross_entropy_of_its_logits():
    dev = torch.device("cuda", 0)
    h = torch.cuda.current_stream().cuda_stream
    step = TrainingStepGemms(SHAPE, dev, micro_batches=1)
    step.run_step(h)
    torch.cuda.synchronize()
    T, books, size = SHAPE.tokens, SHAPE.codebooks, SHAPE.codebook_size
    # Recompute the logits of the last forward (the step overwrote them with the gradient) through the head GEMM.
    args = step.forward_plan[-1][2]
    assert _ffi.load().snb_gemm(h, ctypes.byref(args)) == _ffi.OK
    torch.cuda.synchronize()
    logits = step.logits.float().cpu().numpy().reshape(T, books * size)
    targets = step.targets[0].cpu().numpy().astype(np.uint32)
    losses = np.zeros(T, np.float32)
    grad = np.zeros(T * books * size, np.float32)
    expected = []
    for c in range(books):
        o.cross_entropy(logits.reshape(-1), targets, books * size, c * size, size, books, c, step.grad_scale,
                        losses, grad)
        expected.append(float(losses.astype(np.float64).sum()))
    got = step.loss_sums[0].cpu().numpy().astype(np.float64)
    assert np.allclose(got, expected, rtol=1e-4)


def test_a_captured_micro_batch_replays_the_same_gradients():
    # The step's launches (GEMMs, split-K zeroing, the loss kernel) captured into a CUDA graph: one replay gives the
    # gradients and loss of one run() (to f32 rounding: split-K partials land in arrival order).
    dev = torch.device("cuda", 0)
    h = torch.cuda.current_stream().cuda_stream
    step = TrainingStepGemms(SHAPE, dev, micro_batches=1)
    step.run_step(h)   # first run: per-device set-up outside the capture
    torch.cuda.synchronize()
    ref = _grads(step)
    ref_loss = step.loss_sums.clone()
    graph = step.capture(0)
    step.zero_grads()
    graph.replay()
    torch.cuda.synchronize()
    for a, b in zip(_grads(step), ref):
        assert _rel(a, b) < 1e-6
    assert torch.allclose(step.loss_sums, ref_loss, rtol=1e-6)
