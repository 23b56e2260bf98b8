"""The deterministic mode of the tensor-core GEMM (SNB_GEMM_DETERMINISTIC / snb_set_deterministic): split-K partial
sums reach the output in a fixed order, so a weight gradient computed twice from the same inputs is bit-identical,
as the reference's fixed-order f32 sum is (crates/staleynet-cuda/src/reference.rs:18-38); the result still matches
the default mode and the oracle within the usual tolerances."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import oracle as o  # noqa: E402
from staleynet_b200 import _ffi  # noqa: E402
from staleynet_b200.matmul import Gpu, MatmulKernel, MatmulSpec  # noqa: E402

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def gpu():
    return Gpu(0)


def _rel(a, b):
    return (torch.linalg.vector_norm((a - b).double()) / torch.linalg.vector_norm(b.double())).item()


@pytest.mark.parametrize("accumulate", [True, False])
def test_config2_weight_gradient_is_bit_identical_between_runs(gpu, accumulate):
    # BASELINE config 2's QKV weight gradient: dW[512, 1536] (+)= X^T dY over 16,384 tokens, which the kernel splits
    # along K (few output tiles, long K).
    T, i, out = 16384, 512, 1536
    g = torch.Generator(device="cuda").manual_seed(3)
    x = torch.randn(T, i, device="cuda", generator=g).bfloat16()
    dy = torch.randn(T, out, device="cuda", generator=g).bfloat16()
    c0 = torch.randn(i, out, device="cuda", generator=g)
    spec = MatmulSpec.new(i, out, T).left_transposed()
    if accumulate:
        spec = spec.accumulate()
    results = []
    for det in (True, True, True, False):
        c = c0.clone()
        gpu.gemm(spec, x, dy, c, deterministic=det)
        assert _ffi.last_path() in _ffi.TENSOR_CORE_PATHS
        results.append(c)
    torch.cuda.synchronize()
    assert torch.equal(results[0], results[1]) and torch.equal(results[0], results[2])
    assert _rel(results[0], results[3]) < 1e-5


def test_deterministic_split_k_matches_the_oracle(gpu):
    # bf16-rounded inputs, so the oracle's f32 loop and the tensor core differ only in summation order.
    M, N, K = 256, 512, 8192
    left = o.lcg_values(K * M, 11)    # stored [K, M]: the left operand read transposed, as in dW
    right = o.lcg_values(K * N, 12)
    initial = o.lcg_values(M * N, 13)
    lb, _ = o.round_bf16(left)
    rb, _ = o.round_bf16(right)
    spec = MatmulSpec.new(M, N, K).left_transposed().accumulate().scaled(0.5)
    p = spec.product()
    expected = initial.copy()
    o.matmul(o.product(M, N, K, (p.left.row_stride, p.left.col_stride, 0), (p.right.row_stride, p.right.col_stride, 0),
                       0, 0.5, True), 1, lb, rb, expected)
    c = torch.from_numpy(initial).cuda()
    gpu.gemm(spec, torch.from_numpy(left).cuda().bfloat16(), torch.from_numpy(right).cuda().bfloat16(), c,
             deterministic=True)
    got = c.cpu().numpy()
    assert o.relative_error(expected, got) <= 2e-5 * max(1.0, (K / 1024) ** 0.5)


def test_thread_switch_makes_the_f32_drop_in_deterministic(gpu):
    # snb_set_deterministic covers snb_matmul (the reference's f32 Gpu::matmul, TF32 tensor cores), which has no
    # flags argument: an overwritten dW computed twice is bit-identical and within the TF32 tolerance.
    M, N, K = 384, 768, 16384
    g = torch.Generator(device="cuda").manual_seed(5)
    x = torch.randn(K, M, device="cuda", generator=g)
    dy = torch.randn(K, N, device="cuda", generator=g)
    spec = MatmulSpec.new(M, N, K).left_transposed()
    lib = _ffi.load()
    previous = lib.snb_set_deterministic(1)
    try:
        gpu.matmul_kernel = MatmulKernel.TENSOR_CORE
        outs = []
        for _ in range(2):
            c = torch.full((M, N), 7.0, device="cuda")
            gpu.matmul(spec, x, dy, c)
            outs.append(c)
        torch.cuda.synchronize()
    finally:
        lib.snb_set_deterministic(previous)
    assert torch.equal(outs[0], outs[1])
    exact = x.double().t() @ dy.double()
    assert _rel(outs[0], exact) < 2e-3
