"""GPU parity: every product through the C ABI against the CPU oracle (a restatement of reference::matmul,
crates/staleynet-cuda/src/reference.rs:18-38) on the same seeded inputs.

The first test mirrors the reference's `matmul_matches_reference_for_every_storage_and_kernel`
(crates/staleynet-cuda/tests/kernels_match_reference.rs:55-91): ragged sizes x batch {1, 3} x the four storage
combinations, scale 0.7, accumulating into a random initial output, LCG inputs with seeds 1/2/3, and the
reference's error metric max|delta|/max|expected| against each kernel's tolerance (1e-5 f32, 2e-3 TF32; 1e-2 bf16).
Further tests cover shapes the tcgen05/TMA kernel takes (asserting it ran), split-K, the BASELINE model shapes,
the fused epilogues and the softmax kernels.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import oracle as o  # noqa: E402
from staleynet_b200 import _ffi  # noqa: E402
from staleynet_b200.matmul import BatchStrides, Gpu, MatmulKernel, MatmulSpec, OperandTooSmall  # noqa: E402

pytestmark = pytest.mark.gpu

REFERENCE_SIZES = [(1, 1, 1), (17, 33, 9), (64, 48, 70), (5, 129, 31), (130, 197, 100)]
# Sizes whose strides suit TMA (16-byte multiples for f32 and bf16), with ragged tile edges.
TMA_SIZES = [(128, 256, 64), (130, 200, 104), (257, 264, 136), (64, 64, 64), (300, 72, 520), (1, 128, 64)]
KERNELS = [MatmulKernel.BLOCKED, MatmulKernel.TENSOR_CORE, MatmulKernel.BF16_TENSOR_CORE]


@pytest.fixture(scope="module")
def gpu():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return Gpu(0)


def variants(rows, cols, inner, batch):
    strides = BatchStrides(count=batch, left=rows * inner, right=inner * cols, output=rows * cols)
    base = MatmulSpec.new(rows, cols, inner).batched(strides).scaled(0.7).accumulate()
    return [base, base.left_transposed(), base.right_transposed(), base.left_transposed().right_transposed()]


def expected_product(spec, left, right, initial):
    out = initial.copy()
    o.matmul(to_oracle(spec), spec.batch.count, left, right, out)
    return out


def to_oracle(spec):
    p = spec.product()
    return o.product(p.rows, p.cols, p.inner, (p.left.row_stride, p.left.col_stride, p.left.batch_stride),
                     (p.right.row_stride, p.right.col_stride, p.right.batch_stride), p.output_batch_stride,
                     p.scale, bool(p.accumulate))


def run_on_gpu(gpu, kernel, spec, left, right, initial):
    gpu.matmul_kernel = kernel
    dtype = torch.bfloat16 if kernel is MatmulKernel.BF16_TENSOR_CORE else torch.float32
    lt = torch.from_numpy(left).cuda().to(dtype)
    rt = torch.from_numpy(right).cuda().to(dtype)
    out = torch.from_numpy(initial).cuda()
    gpu.matmul(spec, lt, rt, out)
    path = _ffi.last_path()
    torch.cuda.synchronize()
    return out.cpu().numpy(), path


def tma_eligible(spec, esize):
    p = spec.product()
    unit = 16 // esize
    a_ld = p.left.row_stride if p.left.col_stride == 1 else p.left.col_stride
    b_ld = p.right.col_stride if p.right.row_stride == 1 else p.right.row_stride
    ok = a_ld % unit == 0 and b_ld % unit == 0 and p.cols % 4 == 0
    if spec.batch.count > 1:
        ok = ok and spec.batch.left % unit == 0 and spec.batch.right % unit == 0 and spec.batch.output % 4 == 0
    return ok and p.rows > 1 and p.inner > 1 and p.cols > 1


@pytest.mark.parametrize("rows,cols,inner", REFERENCE_SIZES + TMA_SIZES)
@pytest.mark.parametrize("batch", [1, 3])
def test_matmul_matches_reference_for_every_storage_and_kernel(gpu, rows, cols, inner, batch):
    for spec in variants(rows, cols, inner, batch):
        left = o.lcg_values(batch * rows * inner, 1)
        right = o.lcg_values(batch * inner * cols, 2)
        initial = o.lcg_values(batch * rows * cols, 3)
        expected = expected_product(spec, left, right, initial)
        for kernel in KERNELS:
            actual, path = run_on_gpu(gpu, kernel, spec, left, right, initial)
            error = o.relative_error(expected, actual)
            assert error < kernel.tolerance(), f"{kernel} {spec}: relative error {error}"
            if kernel is MatmulKernel.BLOCKED:
                assert path == _ffi.PATH_SIMT
            elif (rows, cols, inner) in TMA_SIZES:
                esize = 2 if kernel is MatmulKernel.BF16_TENSOR_CORE else 4
                if tma_eligible(spec, esize):
                    assert path in _ffi.TENSOR_CORE_PATHS, f"{kernel} {spec} did not take the tensor-core path"
    gpu.device_status()


@pytest.mark.parametrize("lt,rt", [(False, False), (True, False), (False, True), (True, True)])
def test_bf16_tensor_core_is_exact_up_to_summation_order(gpu, lt, rt):
    """Against the oracle on the same bf16-rounded inputs the only difference left is the f32 summation order."""
    rows, cols, inner, batch = 264, 264, 136, 2  # every stride a multiple of 16 bytes in every storage
    spec = variants(rows, cols, inner, batch)[(1 if lt else 0) + (2 if rt else 0)]
    left, _ = o.round_bf16(o.lcg_values(batch * rows * inner, 4))
    right, _ = o.round_bf16(o.lcg_values(batch * inner * cols, 5))
    initial = o.lcg_values(batch * rows * cols, 6)
    expected = expected_product(spec, left, right, initial)
    actual, path = run_on_gpu(gpu, MatmulKernel.BF16_TENSOR_CORE, spec, left, right, initial)
    assert path in _ffi.TENSOR_CORE_PATHS
    assert o.relative_error(expected, actual) < 2e-5


def test_tf32_rounding_of_the_tensor_core_path(gpu):
    """The TF32 path rounds inputs to 10 mantissa bits: its error against RNA-rounded inputs is at summation
    level, far below its error against the unrounded f32 product."""
    rows, cols, inner = 256, 256, 512
    spec = MatmulSpec.new(rows, cols, inner)
    left = o.lcg_values(rows * inner, 7)
    right = o.lcg_values(inner * cols, 8)
    zero = np.zeros(rows * cols, np.float32)
    actual, path = run_on_gpu(gpu, MatmulKernel.TENSOR_CORE, spec, left, right, zero)
    assert path in _ffi.TENSOR_CORE_PATHS
    exact = expected_product(spec, left, right, zero)
    rounded = expected_product(spec, o.round_tf32(left), o.round_tf32(right), zero)
    err_exact = o.relative_error(exact, actual)
    err_rounded = o.relative_error(rounded, actual)
    assert err_exact < MatmulKernel.TENSOR_CORE.tolerance()
    assert err_rounded < 1e-4, f"tf32 inputs are not round-to-nearest: {err_rounded} vs {err_exact}"


@pytest.mark.parametrize("case", ["dW_split_k", "dW_overwrite_split_k", "dX", "fwd_head_like"])
def test_model_shaped_products(gpu, case):
    """Linear forward / backward layouts (linear.rs:43-63) at reduced token counts; dW has K = tokens, which
    takes the split-K reduce-add path."""
    T, w, out = 4096, 256, 768
    if case == "dW_split_k":
        spec = MatmulSpec.new(w, out, T).left_transposed().accumulate()  # dW += X^T dY
        shapes = (T * w, T * out, w * out)
    elif case == "dW_overwrite_split_k":
        spec = MatmulSpec.new(w, out, T).left_transposed()
        shapes = (T * w, T * out, w * out)
    elif case == "dX":
        spec = MatmulSpec.new(T, w, out).right_transposed()  # dX = dY W^T
        shapes = (T * out, w * out, T * w)
    else:
        spec = MatmulSpec.new(2048, 4096, 256)
        shapes = (2048 * 256, 256 * 4096, 2048 * 4096)
    left = o.lcg_values(shapes[0], 11)
    right = o.lcg_values(shapes[1], 12)
    initial = o.lcg_values(shapes[2], 13)
    expected = initial.copy()
    o.matmul_rows(to_oracle(spec), 1, left, right, expected, 0, spec.rows)
    for kernel in (MatmulKernel.TENSOR_CORE, MatmulKernel.BF16_TENSOR_CORE):
        actual, path = run_on_gpu(gpu, kernel, spec, left, right, initial)
        assert path in _ffi.TENSOR_CORE_PATHS
        assert o.relative_error(expected, actual) < kernel.tolerance()
        assert o.relative_frobenius(expected, actual) < (2e-3 if kernel is MatmulKernel.TENSOR_CORE else 1e-2)
    gpu.device_status()


def test_seeded_baseline_inputs_within_north_star_tolerance(gpu):
    """BASELINE config-1 inputs (X~N(0,1), W~N(0, 1/sqrt(256)) via the reference's SplitMix64, seed 0) on the
    QKV forward shape: relative Frobenius error <= 1e-2 in bf16 and <= 2e-3 in tf32 against the f32 CPU path."""
    T, w = 4096, 256
    rng = o.Random(0)
    x = rng.normals(T * w)
    wt = rng.normals(w * 3 * w, std=1.0 / np.sqrt(256.0))
    spec = MatmulSpec.new(T, 3 * w, w)
    zero = np.zeros(T * 3 * w, np.float32)
    expected = zero.copy()
    o.matmul_rows(to_oracle(spec), 1, x, wt, expected, 0, T)
    for kernel, tol in ((MatmulKernel.TENSOR_CORE, 2e-3), (MatmulKernel.BF16_TENSOR_CORE, 1e-2)):
        actual, _ = run_on_gpu(gpu, kernel, spec, x, wt, zero)
        assert o.relative_frobenius(expected, actual) <= tol


def test_batched_attention_products_match_the_reference_layouts(gpu):
    """The batched QK^T / P.V products of CausalSelfAttention::forward (attention.rs:206-213) with the fp32
    causal softmax between them, against the oracle."""
    B, H, S, d = 2, 3, 136, 64
    count = B * H
    q = o.lcg_values(count * S * d, 21)
    k = o.lcg_values(count * S * d, 22)
    v = o.lcg_values(count * S * d, 23)
    scores_spec = MatmulSpec.new(S, S, d).right_transposed().batched(BatchStrides(count, S * d, S * d, S * S))
    mix_spec = MatmulSpec.new(S, d, S).batched(BatchStrides(count, S * S, S * d, S * d))
    scale = 1.0 / np.sqrt(d)

    exp_scores = np.zeros(count * S * S, np.float32)
    o.matmul(to_oracle(scores_spec), count, q, k, exp_scores)
    o.causal_softmax(exp_scores, S, S, scale, 0)
    exp_ctx = np.zeros(count * S * d, np.float32)
    o.matmul(to_oracle(mix_spec), count, exp_scores, v, exp_ctx)

    gpu.matmul_kernel = MatmulKernel.TENSOR_CORE
    qt, kt, vt = (torch.from_numpy(a).cuda() for a in (q, k, v))
    scores = torch.zeros(count * S, S, device="cuda")
    gpu.matmul(scores_spec, qt, kt, scores)
    assert _ffi.last_path() in _ffi.TENSOR_CORE_PATHS
    gpu.causal_softmax(scores, S, scale, 0)
    ctx = torch.zeros(count * S * d, device="cuda")
    gpu.matmul(mix_spec, scores, vt, ctx)
    assert _ffi.last_path() in _ffi.TENSOR_CORE_PATHS
    torch.cuda.synchronize()
    assert o.relative_error(exp_scores, scores.cpu().numpy().ravel()) < 2e-3
    assert o.relative_error(exp_ctx, ctx.cpu().numpy()) < 2e-3


@pytest.mark.parametrize("offset", [0, 5])
def test_causal_softmax_matches_reference(gpu, offset):
    rows, queries, keys = 6 * 37, 37, 70
    scores = o.lcg_values(rows * keys, 31) * 4
    expected = scores.copy()
    o.causal_softmax(expected, queries, keys, 0.125, offset)
    t = torch.from_numpy(scores.reshape(rows, keys)).cuda()
    gpu.causal_softmax(t, queries, 0.125, offset)
    torch.cuda.synchronize()
    assert o.relative_error(expected, t.cpu().numpy()) < 1e-5
    masked = np.triu(np.ones((queries, keys), bool), k=offset + 1)
    assert np.all(t.cpu().numpy().reshape(6, queries, keys)[:, masked] == 0)


def test_softmax_backward_matches_reference(gpu):
    rows, cols = 37, 70
    p = np.abs(o.lcg_values(rows * cols, 41))
    p /= p.reshape(rows, cols).sum(axis=1, keepdims=True).repeat(cols, axis=1).ravel()
    p = p.astype(np.float32)
    g = o.lcg_values(rows * cols, 42)
    expected = g.copy()
    o.softmax_backward(p, expected, cols)
    pt = torch.from_numpy(p.reshape(rows, cols)).cuda()
    gt = torch.from_numpy(g.reshape(rows, cols)).cuda()
    gpu.softmax_backward(pt, gt)
    torch.cuda.synchronize()
    assert o.relative_error(expected, gt.cpu().numpy()) < 1e-4


@pytest.mark.parametrize("out_dtype", ["f32", "bf16"])
def test_fused_linear_forward_bias_gelu_and_residual(gpu, out_dtype):
    """snb_gemm = Linear::forward (+bias) -> gelu_forward with the pre-activation kept (feed_forward.rs:55-59),
    and the residual add of block.rs:188, against the oracle composed step by step."""
    T, w, f = 384, 256, 1024
    x = o.lcg_values(T * w, 51)
    w1 = o.lcg_values(w * f, 52) * 0.1
    b1 = o.lcg_values(f, 53)
    res = o.lcg_values(T * f, 54)
    spec = MatmulSpec.new(T, f, w)
    xb, _ = o.round_bf16(x)
    wb, _ = o.round_bf16(w1)
    pre = np.zeros(T * f, np.float32)
    o.matmul(to_oracle(spec), 1, xb, wb, pre)
    pre = pre + np.tile(b1, T)
    out_exp = o.gelu(pre) + res
    odt = torch.bfloat16 if out_dtype == "bf16" else torch.float32
    xt = torch.from_numpy(x).cuda().to(torch.bfloat16)
    wt = torch.from_numpy(w1).cuda().to(torch.bfloat16)
    bt = torch.from_numpy(b1).cuda()
    rt = torch.from_numpy(res).cuda().to(odt)
    out = torch.empty(T * f, device="cuda", dtype=odt)
    pre_t = torch.empty(T * f, device="cuda", dtype=odt)
    gpu.gemm(spec, xt, wt, out, bias=bt, activation=_ffi.ACTIVATION_GELU, pre_activation=pre_t, residual=rt)
    assert _ffi.last_path() in _ffi.TENSOR_CORE_PATHS
    torch.cuda.synchronize()
    if out_dtype == "bf16":
        res_used = rt.float().cpu().numpy()
        out_exp = o.gelu(pre) + res_used
    tol = 1e-2 if out_dtype == "bf16" else 1e-4
    assert o.relative_error(pre, pre_t.float().cpu().numpy()) < tol
    assert o.relative_error(out_exp, out.float().cpu().numpy()) < tol


def test_fused_gelu_backward_epilogue(gpu):
    """dH = (dY W2^T) * gelu'(pre): project.backward's dX product fused with gelu_backward (feed_forward.rs:72-74)."""
    T, w, f = 256, 256, 512
    dy = o.lcg_values(T * w, 61)
    w2 = o.lcg_values(f * w, 62) * 0.1
    pre = o.lcg_values(T * f, 63) * 3
    spec = MatmulSpec.new(T, f, w).right_transposed()
    dyb, _ = o.round_bf16(dy)
    w2b, _ = o.round_bf16(w2)
    dh = np.zeros(T * f, np.float32)
    o.matmul(to_oracle(spec), 1, dyb, w2b, dh)
    expected = dh * o.gelu_derivative(pre)
    out = torch.empty(T * f, device="cuda")
    gpu.gemm(spec, torch.from_numpy(dy).cuda().bfloat16(), torch.from_numpy(w2).cuda().bfloat16(), out,
             activation=_ffi.ACTIVATION_GELU_GRAD, gelu_input=torch.from_numpy(pre).cuda())
    assert _ffi.last_path() in _ffi.TENSOR_CORE_PATHS
    torch.cuda.synchronize()
    assert o.relative_error(expected, out.cpu().numpy()) < 1e-4


@pytest.mark.parametrize("kind", ["gelu_grad", "bias_residual"])
@pytest.mark.parametrize("rows,cols,inner,batch", [(384, 520, 256, 1), (384, 520, 2048, 1), (200, 136, 96, 1),
                                                   (130, 72, 64, 1), (260, 264, 128, 2)])
def test_bf16_auxiliary_input_staged_by_tma(gpu, kind, rows, cols, inner, batch):
    """bf16 outputs whose one bf16 auxiliary input (the GELU input of project.backward's dX product, or a block's
    residual) is TMA-loaded into the epilogue's staging boxes: single-CTA and CTA-pair tiles, ragged tile edges
    (rows, and columns not a multiple of the 64-column chunk), and a batch of two."""
    T, n, k = rows, cols, inner
    x = o.lcg_values(batch * T * k, 81)
    w = o.lcg_values(batch * k * n, 82) * 0.05
    b = o.lcg_values(n, 83)
    aux = o.lcg_values(batch * T * n, 84) * 2
    xb, _ = o.round_bf16(x)
    wb, _ = o.round_bf16(w)
    auxb, _ = o.round_bf16(aux)
    spec = MatmulSpec.new(T, n, k)
    if batch > 1:
        spec = spec.batched(BatchStrides(count=batch, left=T * k, right=k * n, output=T * n))
    acc = np.zeros(batch * T * n, np.float32)
    o.matmul(to_oracle(spec), batch, xb, wb, acc)
    xt, wt = torch.from_numpy(x).cuda().bfloat16(), torch.from_numpy(w).cuda().bfloat16()
    at = torch.from_numpy(aux).cuda().bfloat16()
    out = torch.empty(batch * T * n, device="cuda", dtype=torch.bfloat16)
    if kind == "gelu_grad":
        gpu.gemm(spec, xt, wt, out, activation=_ffi.ACTIVATION_GELU_GRAD, gelu_input=at)
        expected = acc * o.gelu_derivative(auxb)
    else:
        gpu.gemm(spec, xt, wt, out, bias=torch.from_numpy(b).cuda(), residual=at)
        expected = acc + np.tile(b, batch * T) + auxb
    assert _ffi.last_path() in _ffi.TENSOR_CORE_PATHS
    if k >= 2048:
        assert _ffi.last_path() == _ffi.PATH_TENSOR_CORE_PAIR
    torch.cuda.synchronize()
    assert o.relative_error(expected, out.float().cpu().numpy()) < 1e-2
    gpu.device_status()


@pytest.mark.parametrize("out_dtype", ["f32", "bf16"])
@pytest.mark.parametrize("rows,cols,inner,batch", [(130, 264, 104, 1), (257, 520, 256, 3), (300, 392, 2048, 1)])
def test_overwritten_outputs_at_ragged_tile_edges(gpu, out_dtype, rows, cols, inner, batch):
    """Products that overwrite C (no accumulation) on 256-column tiles, whose epilogue warps write the staged boxes
    to global memory themselves: ragged rows and columns, batches, single-CTA and CTA-pair tiles; C's other
    elements (past each matrix's end in the batch stride) stay untouched."""
    T, n, k = rows, cols, inner
    gap = 48  # output batch stride = T * n + gap
    x = o.lcg_values(batch * T * k, 91)
    w = o.lcg_values(batch * k * n, 92) * 0.05
    xb, _ = o.round_bf16(x)
    wb, _ = o.round_bf16(w)
    spec = MatmulSpec.new(T, n, k).batched(BatchStrides(count=batch, left=T * k, right=k * n, output=T * n + gap))
    odt = torch.bfloat16 if out_dtype == "bf16" else torch.float32
    out = torch.full((batch * (T * n + gap),), 7.0, device="cuda", dtype=odt)
    expected = np.full(batch * (T * n + gap), 7.0, np.float32)
    o.matmul(to_oracle(spec), batch, xb, wb, expected)
    gpu.gemm(spec, torch.from_numpy(x).cuda().bfloat16(), torch.from_numpy(w).cuda().bfloat16(), out)
    assert _ffi.last_path() in _ffi.TENSOR_CORE_PATHS
    torch.cuda.synchronize()
    got = out.float().cpu().numpy()
    tol = 1e-2 if out_dtype == "bf16" else 1e-5
    assert o.relative_error(expected, got) < tol
    for b in range(batch):  # the gaps between matrices keep their initial value exactly
        assert np.all(got[b * (T * n + gap) + T * n:(b + 1) * (T * n + gap)] == 7.0)
    gpu.device_status()


def test_undersized_operands_raise_like_the_reference(gpu):
    gpu.matmul_kernel = MatmulKernel.TENSOR_CORE
    a = torch.zeros(23, device="cuda")
    b = torch.zeros(30, device="cuda")
    c = torch.zeros(20, device="cuda")
    with pytest.raises(OperandTooSmall, match="left operand too small"):
        gpu.matmul(MatmulSpec.new(4, 5, 6), a, b, c)
    gpu.device_status()


def test_bounded_wait_gives_up_and_the_context_stays_usable(gpu):
    """Failure detection on the device: a wait that nothing completes returns after its limit with an error status
    the host reads, instead of hanging; the next product still runs correctly."""
    import ctypes

    lib = _ffi.load()
    handle = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    gpu.device_status()  # start clean
    assert lib.snb_selftest_bounded_wait(handle, 20_000_000) == _ffi.OK
    assert lib.snb_device_status() == _ffi.ERR_DEVICE_TIMEOUT
    assert lib.snb_device_status() == _ffi.OK  # reading clears it
    spec = MatmulSpec.new(128, 256, 64)
    left, right = o.lcg_values(128 * 64, 1), o.lcg_values(64 * 256, 2)
    zero = np.zeros(128 * 256, np.float32)
    actual, path = run_on_gpu(gpu, MatmulKernel.TENSOR_CORE, spec, left, right, zero)
    assert path in _ffi.TENSOR_CORE_PATHS
    assert o.relative_error(expected_product(spec, left, right, zero), actual) < MatmulKernel.TENSOR_CORE.tolerance()
    gpu.device_status()


PAIR_SIZES = [(264, 264, 2056), (520, 392, 2048), (1024, 768, 4096)]  # 16-byte strides, ragged tiles


@pytest.mark.parametrize("rows,cols,inner", PAIR_SIZES)
@pytest.mark.parametrize("batch", [1, 3])
def test_cta_pair_kernel_matches_reference_for_every_storage(gpu, rows, cols, inner, batch):
    """Long-K products run on CTA pairs (cta_group::2): every storage, batched, scale + accumulate, against the
    oracle on the same bf16-rounded inputs (summation order only) and on f32 inputs in tf32."""
    for spec in variants(rows, cols, inner, batch):
        left = o.lcg_values(batch * rows * inner, 1)
        right = o.lcg_values(batch * inner * cols, 2)
        initial = o.lcg_values(batch * rows * cols, 3)
        lb, _ = o.round_bf16(left)
        rb, _ = o.round_bf16(right)
        expected = initial.copy()
        o.matmul_rows(to_oracle(spec), batch, lb, rb, expected, 0, rows)
        actual, path = run_on_gpu(gpu, MatmulKernel.BF16_TENSOR_CORE, spec, lb, rb, initial)
        assert path == _ffi.PATH_TENSOR_CORE_PAIR, f"{spec} did not run on CTA pairs"
        assert o.relative_error(expected, actual) < 2e-5, spec
        expected = initial.copy()
        o.matmul_rows(to_oracle(spec), batch, left, right, expected, 0, rows)
        actual, path = run_on_gpu(gpu, MatmulKernel.TENSOR_CORE, spec, left, right, initial)
        assert path == _ffi.PATH_TENSOR_CORE_PAIR
        assert o.relative_error(expected, actual) < MatmulKernel.TENSOR_CORE.tolerance(), spec
    gpu.device_status()


@pytest.mark.parametrize("epilogue", ["bias_residual_bf16", "gelu_pre_bf16", "gelu_grad_f32", "split_k_overwrite"])
def test_cta_pair_kernel_fused_epilogues(gpu, epilogue):
    """The pair kernel's epilogue (the single-CTA code on each CTA's 128 rows) with every fused option."""
    T, n, k = 384, 520, 2048
    x = o.lcg_values(T * k, 71)
    w = o.lcg_values(k * n, 72) * 0.05
    b = o.lcg_values(n, 73)
    res = o.lcg_values(T * n, 74)
    gin = o.lcg_values(T * n, 75) * 2
    xb, _ = o.round_bf16(x)
    wb, _ = o.round_bf16(w)
    spec = MatmulSpec.new(T, n, k)
    acc = np.zeros(T * n, np.float32)
    o.matmul_rows(to_oracle(spec), 1, xb, wb, acc, 0, T)
    xt, wt = torch.from_numpy(x).cuda().bfloat16(), torch.from_numpy(w).cuda().bfloat16()
    if epilogue == "bias_residual_bf16":
        rt = torch.from_numpy(res).cuda().bfloat16()
        out = torch.empty(T * n, device="cuda", dtype=torch.bfloat16)
        gpu.gemm(spec, xt, wt, out, bias=torch.from_numpy(b).cuda(), residual=rt)
        expected = acc + np.tile(b, T) + rt.float().cpu().numpy()
        tol = 1e-2
    elif epilogue == "gelu_pre_bf16":
        out = torch.empty(T * n, device="cuda", dtype=torch.bfloat16)
        pre = torch.empty(T * n, device="cuda", dtype=torch.bfloat16)
        gpu.gemm(spec, xt, wt, out, bias=torch.from_numpy(b).cuda(), activation=_ffi.ACTIVATION_GELU,
                 pre_activation=pre)
        expected = o.gelu(acc + np.tile(b, T))
        assert o.relative_error(acc + np.tile(b, T), pre.float().cpu().numpy()) < 1e-2
        tol = 1e-2
    elif epilogue == "gelu_grad_f32":
        out = torch.empty(T * n, device="cuda")
        gpu.gemm(spec, xt, wt, out, activation=_ffi.ACTIVATION_GELU_GRAD, gelu_input=torch.from_numpy(gin).cuda())
        expected = acc * o.gelu_derivative(gin)
        tol = 1e-4
    else:
        spec = MatmulSpec.new(n, T, k)  # rows 520 x cols 384: few tiles, K split across the grid
        acc = np.zeros(n * T, np.float32)
        wt2 = torch.from_numpy(o.lcg_values(n * k, 76)).cuda().bfloat16()
        xt2 = torch.from_numpy(o.lcg_values(k * T, 77)).cuda().bfloat16()
        o.matmul_rows(to_oracle(spec), 1, wt2.float().cpu().numpy().ravel(), xt2.float().cpu().numpy().ravel(), acc,
                      0, n)
        out = torch.full((n * T,), 5.0, device="cuda")
        gpu.gemm(spec, wt2, xt2, out)
        expected = acc
        tol = 2e-5
    assert _ffi.last_path() == _ffi.PATH_TENSOR_CORE_PAIR
    torch.cuda.synchronize()
    assert o.relative_error(expected, out.float().cpu().numpy()) < tol
    gpu.device_status()


@pytest.mark.parametrize("epilogue", ["bias", "bias_gelu_pre", "bias_residual"])
@pytest.mark.parametrize("rows,cols,inner", [(8192, 2304, 768), (1000, 648, 256), (16392, 776, 64)])
def test_short_k_bias_products_stage_the_bias_in_shared_memory(gpu, epilogue, rows, cols, inner):
    """Short-K bf16 products with a bias and a bf16 output (the forward linears: qkv, expand, output, head) run on
    CTA pairs whose producer copies each tile's bias into one of two shared-memory buffers while the epilogue of the
    previous tile on that buffer finishes. Every staging mode (plain, GELU with the pre-activation kept, residual by
    TMA into the staging boxes), ragged rows and columns, and enough tiles per CTA pair (up to ~4) that both buffers
    are reused; a distinct bias per column, so a tile reading another tile's buffer shows."""
    T, n, k = rows, cols, inner
    x = o.lcg_values(T * k, 91)
    w = o.lcg_values(k * n, 92) * 0.05
    b = o.lcg_values(n, 93) * 4
    res = o.lcg_values(T * n, 94)
    xb, _ = o.round_bf16(x)
    wb, _ = o.round_bf16(w)
    spec = MatmulSpec.new(T, n, k)
    acc = np.zeros(T * n, np.float32)
    o.matmul(to_oracle(spec), 1, xb, wb, acc)
    xt, wt = torch.from_numpy(x).cuda().bfloat16(), torch.from_numpy(w).cuda().bfloat16()
    bt = torch.from_numpy(b).cuda()
    out = torch.empty(T * n, device="cuda", dtype=torch.bfloat16)
    lin = acc + np.tile(b, T)
    if epilogue == "bias":
        gpu.gemm(spec, xt, wt, out, bias=bt)
        expected = lin
    elif epilogue == "bias_gelu_pre":
        pre = torch.empty(T * n, device="cuda", dtype=torch.bfloat16)
        gpu.gemm(spec, xt, wt, out, bias=bt, activation=_ffi.ACTIVATION_GELU, pre_activation=pre)
        expected = o.gelu(lin)
        torch.cuda.synchronize()
        assert o.relative_error(lin, pre.float().cpu().numpy()) < 1e-2
    else:
        rt = torch.from_numpy(res).cuda().bfloat16()
        gpu.gemm(spec, xt, wt, out, bias=bt, residual=rt)
        expected = lin + rt.float().cpu().numpy()
    assert _ffi.last_path() == _ffi.PATH_TENSOR_CORE_PAIR
    torch.cuda.synchronize()
    got = out.float().cpu().numpy()
    assert o.relative_error(expected, got) < 1e-2
    # Column by column: a tile whose bias came from the wrong buffer is off by a whole bias difference.
    col_err = np.abs(expected.reshape(T, n) - got.reshape(T, n)).max(axis=0)
    assert col_err.max() < 0.05 * max(1.0, float(np.abs(expected).max()))
    gpu.device_status()


GOLDEN = __import__("json").loads((__import__("pathlib").Path(__file__).parent / "golden" / "reference_kats.json").read_text())


@pytest.mark.parametrize("case", GOLDEN["matmul"], ids=lambda c: c["name"])
def test_reference_known_answers_on_the_gpu(gpu, case):
    """The reference's own matmul known answers (reference.rs:177-224) through every arithmetic of the C ABI."""
    b = case["batch"]
    spec = MatmulSpec.new(case["rows"], case["cols"], case["inner"]).scaled(case["scale"]).batched(
        BatchStrides(b["count"], b["left"], b["right"], b["output"]))
    if case["left_transposed"]:
        spec = spec.left_transposed()
    if case["right_transposed"]:
        spec = spec.right_transposed()
    if case["accumulate"]:
        spec = spec.accumulate()
    for kernel in KERNELS:
        actual, _ = run_on_gpu(gpu, kernel, spec, np.array(case["left"], np.float32),
                               np.array(case["right"], np.float32), np.array(case["initial"], np.float32))
        assert actual.tolist() == case["expected"], kernel  # small integers: exact in every arithmetic


@pytest.mark.parametrize("accumulate", [False, True])
def test_empty_inner_dimension(gpu, accumulate):
    """K = 0: the reference's loop leaves sum = 0, so C = scale*0 (overwrite) or C unchanged (accumulate)."""
    spec = MatmulSpec.new(5, 7, 0).scaled(0.5)
    if accumulate:
        spec = spec.accumulate()
    initial = o.lcg_values(35, 9)
    for kernel in KERNELS:
        dtype = torch.bfloat16 if kernel is MatmulKernel.BF16_TENSOR_CORE else torch.float32
        gpu.matmul_kernel = kernel
        out = torch.from_numpy(initial.copy()).cuda()
        gpu.matmul(spec, torch.zeros(1, device="cuda", dtype=dtype), torch.zeros(1, device="cuda", dtype=dtype), out)
        torch.cuda.synchronize()
        expected = initial if accumulate else np.zeros(35, np.float32)
        assert np.array_equal(out.cpu().numpy(), expected)


@pytest.mark.parametrize("budget", [1, 2, 17, 132])
def test_gemm_under_an_sm_budget_computes_the_same_product(gpu, budget):
    # A capped persistent grid (snb_set_sm_budget) walks the same work units with fewer CTAs; the split-K choice may
    # change with the worker count, so the weight gradient is compared within f32 summation-order tolerance.
    g = torch.Generator(device="cuda").manual_seed(21)
    T, i, o = 4096, 256, 768
    x = torch.randn(T, i, device="cuda", generator=g).bfloat16()
    w = torch.randn(i, o, device="cuda", generator=g).bfloat16()
    dy = torch.randn(T, o, device="cuda", generator=g).bfloat16()
    lib = _ffi.load()
    outs = []
    for b in (0, budget):
        previous = lib.snb_set_sm_budget(b)
        try:
            y = torch.empty(T, o, device="cuda", dtype=torch.bfloat16)
            gpu.gemm(MatmulSpec.new(T, o, i), x, w, y)
            dw = torch.zeros(i, o, device="cuda")
            gpu.gemm(MatmulSpec.new(i, o, T).left_transposed().accumulate(), x, dy, dw)
            assert _ffi.last_path() in _ffi.TENSOR_CORE_PATHS or budget == 1
        finally:
            lib.snb_set_sm_budget(previous)
        outs.append((y, dw))
    torch.cuda.synchronize()
    if budget >= 2:
        assert torch.equal(outs[0][0], outs[1][0])   # same kernel, same tiles, no split: the same values
    else:
        # One SM rules out the CTA-pair kernel: the single-CTA tiles may round a few bf16 outputs the other way.
        ry = (torch.linalg.vector_norm((outs[0][0] - outs[1][0]).float()) /
              torch.linalg.vector_norm(outs[0][0].float())).item()
        assert ry < 1e-3
    rel = (torch.linalg.vector_norm(outs[0][1] - outs[1][1]) / torch.linalg.vector_norm(outs[0][1])).item()
    assert rel < 1e-5
