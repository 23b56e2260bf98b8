"""RMSNorm, its fused GEMM prologue, AdamW and the gradient-norm reduction on the GPU, against the oracle's
restatements of the reference (reference.rs:60-98, kernels/optimizer.rs:47-113), mirroring the reference's parity
tests (crates/staleynet-cuda/tests/kernels_match_reference.rs:93-124 and 299-327)."""
import json
from pathlib import Path

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import oracle as o  # noqa: E402
from staleynet_b200 import _ffi  # noqa: E402
from staleynet_b200.matmul import AdamWHyperparameters, Gpu, MatmulSpec  # noqa: E402

pytestmark = pytest.mark.gpu

KATS = json.loads((Path(__file__).parent / "golden" / "reference_kats.json").read_text())


def _cuda(a):
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).cuda()


def test_rms_norm_matches_the_reference_parity_case():
    """kernels_match_reference.rs:93-124: 37x70, epsilon 1e-5, LCG inputs (seeds 4, 5, 6); forward 1e-5,
    backward 1e-4 (max|d|/max|ref|)."""
    rows, cols, eps = 37, 70, 1e-5
    x, g, dy = o.lcg_values(rows * cols, 4), o.lcg_values(cols, 5), o.lcg_values(rows * cols, 6)
    e_out, e_inv = o.rms_norm_forward(x, g, cols, eps)
    e_dx, e_dg = o.rms_norm_backward(dy, x, g, e_inv, cols)
    gpu = Gpu(0)
    out = torch.zeros(rows, cols, device="cuda")
    inv = torch.zeros(rows, device="cuda")
    xt = _cuda(x).view(rows, cols)
    gpu.rms_norm_forward(xt, _cuda(g), out, inv, eps)
    dx = torch.zeros(rows, cols, device="cuda")
    dg = torch.zeros(cols, device="cuda")
    gpu.rms_norm_backward(_cuda(dy).view(rows, cols), xt, _cuda(g), inv, dx, dg)
    torch.cuda.synchronize()
    assert o.relative_error(e_out, out.cpu().numpy().ravel()) < 1e-5
    assert o.relative_error(e_inv, inv.cpu().numpy()) < 1e-5
    assert o.relative_error(e_dx, dx.cpu().numpy().ravel()) < 1e-4
    assert o.relative_error(e_dg, dg.cpu().numpy()) < 1e-4


@pytest.mark.parametrize("case", KATS["rms_norm"], ids=lambda c: c["name"])
def test_rms_norm_known_answers_on_the_gpu(case):
    from test_oracle import _check_entry

    gpu = Gpu(0)
    cols = case["cols"]
    if "output_grad" in case:
        dx = torch.zeros(1, cols, device="cuda")
        dg = torch.zeros(cols, device="cuda")
        gpu.rms_norm_backward(_cuda(case["output_grad"]).view(1, cols), _cuda(case["input"]).view(1, cols),
                              _cuda(case["gain"]), _cuda(case["inv_rms"]), dx, dg)
        torch.cuda.synchronize()
        for v, e in zip(dx.cpu().numpy().ravel(), case["expected_input_grad"]):
            _check_entry(float(v), e)
        for v, e in zip(dg.cpu().numpy(), case["expected_gain_grad"]):
            _check_entry(float(v), e)
    else:
        out = torch.zeros(1, cols, device="cuda")
        inv = torch.zeros(1, device="cuda")
        gpu.rms_norm_forward(_cuda(case["input"]).view(1, cols), _cuda(case["gain"]), out, inv, case["epsilon"])
        torch.cuda.synchronize()
        for v, e in zip(inv.cpu().numpy(), case["expected_inv_rms"]):
            _check_entry(float(v), e)
        for v, e in zip(out.cpu().numpy().ravel(), case["expected_output"]):
            _check_entry(float(v), e)


def test_rms_norm_checks_in_the_reference_order():
    gpu = Gpu(0)
    x = torch.zeros(4, 8, device="cuda")
    with pytest.raises(AssertionError, match="gain length"):
        gpu.rms_norm_forward(x, torch.zeros(7, device="cuda"), torch.zeros(4, 8, device="cuda"),
                             torch.zeros(4, device="cuda"), 1e-5)
    with pytest.raises(AssertionError, match="inv_rms too small"):
        gpu.rms_norm_forward(x, torch.zeros(8, device="cuda"), torch.zeros(4, 8, device="cuda"),
                             torch.zeros(3, device="cuda"), 1e-5)


def test_adamw_matches_the_reference_parity_case():
    """kernels_match_reference.rs:299-327: 300 weights, step 2, moments 0.01 / 0.02; 1e-5."""
    c = KATS["adamw"]
    w, g = o.lcg_values(c["count"], c["parameter_seed"]), o.lcg_values(c["count"], c["gradient_seed"])
    m = np.full(c["count"], c["initial_mean"], np.float32)
    v = np.full(c["count"], c["initial_variance"], np.float32)
    hyper = AdamWHyperparameters(c["learning_rate"], c["beta1"], c["beta2"], c["epsilon"], c["weight_decay"], c["step"])
    pt, mt, vt = _cuda(w), _cuda(m), _cuda(v)
    Gpu(0).adamw_step(pt, _cuda(g), mt, vt, hyper)
    torch.cuda.synchronize()
    e = w.copy()
    o.adamw_step(e, g, m, v, c["learning_rate"], c["beta1"], c["beta2"], c["epsilon"], c["weight_decay"], c["step"])
    assert o.relative_error(e, pt.cpu().numpy()) < 1e-5
    assert o.relative_error(m, mt.cpu().numpy()) < 1e-5 and o.relative_error(v, vt.cpu().numpy()) < 1e-5


def test_sum_of_squares_and_multi_tensor_adamw_with_clipping():
    """Several tensors (one empty, sizes not multiples of the kernel's chunk) in one call; the global norm exceeds
    max_gradient_norm, so every gradient is scaled by max/norm before its update, as AdamW::step
    (model optimizer.rs:125-160) does tensor by tensor."""
    rng = np.random.default_rng(9)
    sizes = [300, 0, 16384 * 3 + 17, 768, 70000]
    decays = [0.1, 0.1, 0.0, 0.1, 0.0]
    host = [(rng.standard_normal(n).astype(np.float32), rng.standard_normal(n).astype(np.float32),
             (rng.standard_normal(n) * 0.01).astype(np.float32), (rng.random(n) * 0.02).astype(np.float32))
            for n in sizes]
    gpu = Gpu(0)
    total = torch.zeros(1, device="cuda", dtype=torch.float64)
    gpu.sum_of_squares(_cuda(host[2][1]), total)
    torch.cuda.synchronize()
    assert abs(total.item() - o.sum_of_squares(host[2][1])) <= 1e-5 * o.sum_of_squares(host[2][1])
    dev = [tuple(_cuda(a) for a in h) for h in host]
    hyper = AdamWHyperparameters(3e-4, 0.9, 0.95, 1e-8, 0.0, 7)
    max_norm = 1.0
    gpu.adamw_step_multi([(p, g, m, v, wd) for (p, g, m, v), wd in zip(dev, decays)], hyper, max_norm, total)
    torch.cuda.synchronize()
    square_sum = sum(o.sum_of_squares(h[1]) for h in host)
    assert abs(total.item() - square_sum) <= 1e-5 * square_sum
    norm = np.float32(np.sqrt(square_sum))
    clip = np.float32(max_norm) / norm if norm > max_norm else np.float32(1.0)
    for (w, g, m, v), (pt, gt, mt, vt), wd in zip(host, dev, decays):
        if w.size == 0:
            continue
        e, em, ev = w.copy(), m.copy(), v.copy()
        o.adamw_step(e, (g * clip).astype(np.float32), em, ev, hyper.learning_rate, hyper.beta1, hyper.beta2,
                     hyper.epsilon, wd, hyper.step)
        assert o.relative_error(e, pt.cpu().numpy()) < 1e-5
        assert o.relative_error(em, mt.cpu().numpy()) < 1e-5 and o.relative_error(ev, vt.cpu().numpy()) < 1e-5


def test_multi_tensor_adamw_on_views_that_are_not_16_byte_aligned():
    """Tensors whose arrays start one element into an allocation take the kernel's scalar path, aligned ones the
    float4 path; both give the reference's per-element update."""
    rng = np.random.default_rng(5)
    sizes, offsets = [1001, 4096, 16384 + 6], [1, 0, 3]
    host = [tuple(rng.standard_normal(n).astype(np.float32) * s for s in (1.0, 1.0, 0.01)) +
            ((rng.random(n) * 0.02).astype(np.float32),) for n in sizes]
    dev = []
    for arrays, off in zip(host, offsets):
        views = []
        for a in arrays:
            buf = torch.zeros(a.size + off, device="cuda")
            buf[off:] = torch.from_numpy(a).cuda()
            views.append(buf[off:])
        dev.append(tuple(views))
    gpu = Gpu(0)
    total = torch.zeros(1, device="cuda", dtype=torch.float64)
    hyper = AdamWHyperparameters(1e-3, 0.9, 0.999, 1e-8, 0.0, 3)
    gpu.adamw_step_multi([(p, g, m, v, 0.01) for p, g, m, v in dev], hyper, 1e9, total)
    torch.cuda.synchronize()
    assert abs(total.item() - sum(o.sum_of_squares(h[1]) for h in host)) <= 1e-5 * total.item()
    for (w, g, m, v), (pt, _, mt, vt) in zip(host, dev):
        e, em, ev = w.copy(), m.copy(), v.copy()
        o.adamw_step(e, g, em, ev, hyper.learning_rate, hyper.beta1, hyper.beta2, hyper.epsilon, 0.01, hyper.step)
        assert o.relative_error(e, pt.cpu().numpy()) < 1e-5
        assert o.relative_error(em, mt.cpu().numpy()) < 1e-5 and o.relative_error(ev, vt.cpu().numpy()) < 1e-5


@pytest.mark.parametrize("rows,cols", [(300, 2304), (200, 513)])
def test_fused_rms_norm_prologue_equals_norm_then_gemm(rows, cols):
    """rms_norm(x) W computed as diag(1/rms) x (diag(g) W): snb_rms_norm_stats + snb_scale_rows + snb_gemm with
    row_scale (the second size takes the SIMT kernel), against the float64 composition; relative Frobenius <= 1e-2
    (bf16 operands), and the unfused bf16 path (normalised rows stored as bf16, then the GEMM) to the same bound."""
    width, eps = 768, 1e-5
    g = torch.Generator(device="cuda")
    g.manual_seed(2)
    x = torch.randn(rows, width, device="cuda", generator=g).bfloat16()
    gain = 1.0 + 0.1 * torch.randn(width, device="cuda", generator=g)
    w = (torch.randn(width, cols, device="cuda", generator=g) / width ** 0.5).bfloat16()
    bias = 0.1 * torch.randn(cols, device="cuda", generator=g)
    gpu = Gpu(0)
    inv = torch.empty(rows, device="cuda")
    gpu.rms_norm_stats(x, eps, inv)
    wg = torch.empty_like(w)
    gpu.scale_rows(gain, w, wg)
    y = torch.empty(rows, cols, device="cuda")
    gpu.gemm(MatmulSpec.new(rows, cols, width), x, wg, y, bias=bias, row_scale=inv)
    xn = torch.empty(rows, width, device="cuda", dtype=torch.bfloat16)
    inv2 = torch.empty(rows, device="cuda")
    gpu.rms_norm_stats(x, eps, inv2, gain=gain, output=xn)
    y2 = torch.empty(rows, cols, device="cuda")
    gpu.gemm(MatmulSpec.new(rows, cols, width), xn, w, y2, bias=bias)
    torch.cuda.synchronize()
    xd = x.double()
    ref = (xd / torch.sqrt((xd * xd).mean(dim=1, keepdim=True) + eps) * gain.double()) @ w.double() + bias.double()
    for got in (y, y2):
        err = (torch.linalg.vector_norm(got.double() - ref) / torch.linalg.vector_norm(ref)).item()
        assert err < 1e-2
    assert torch.allclose(inv, inv2)
    assert _ffi.load().snb_device_status() == _ffi.OK
