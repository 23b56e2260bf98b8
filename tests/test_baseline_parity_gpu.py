"""Parity at the BASELINE sizes through the C ABI, with inputs from the reference's generator (Random::new(0),
random.rs:27-70, drawn on the device): every linear GEMM of one decoder block in full tensors at configs 1 and 2
(the tighter same-operand bar on first, middle and last row blocks), and sampled full output rows of every linear
GEMM shape and of the 768 -> 16x1024 head at config 3.

Two bars per product, as the north star states them for bf16:
  - against the CPU loop (reference::matmul, reference.rs:18-38) on the same bf16-rounded operands, which differs
    from the tensor core only in the order of its f32 sums: max|delta| / max|expected| <= 2e-5 * max(1, sqrt(K/1024))
    (the sequential f32 sum's rounding grows like sqrt(K); K reaches 65,536 in config 3's dW products);
  - against the fp32 CPU path on the unrounded f32 operands: relative Frobenius <= 1e-2."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import oracle as o  # noqa: E402
from staleynet_b200 import _ffi  # noqa: E402
from staleynet_b200.matmul import DeviceRandom, Gpu, MatmulKernel, MatmulSpec  # noqa: E402

pytestmark = pytest.mark.gpu

CONFIGS = {1: (4096, 256), 2: (16384, 512), 3: (65536, 768)}   # tokens per step, width


@pytest.fixture(scope="module")
def gpu():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    g = Gpu(0)
    g.matmul_kernel = MatmulKernel.BF16_TENSOR_CORE
    return g


def block_gemms(T: int, w: int):
    """(name, M, N, K, left transposed, right transposed, operand stds) of one block's linear GEMMs
    (linear.rs:43-63): forward Y = X W, dX = dY W^T, dW = X^T dY."""
    out = []
    for name, i, o_ in (("qkv", w, 3 * w), ("output", w, w), ("expand", w, 4 * w), ("project", 4 * w, w)):
        ws = 1.0 / np.sqrt(w)
        out.append((f"{name}.fwd", T, o_, i, False, False, (1.0, ws)))
        out.append((f"{name}.dX", T, i, o_, False, True, (1.0, ws)))
        out.append((f"{name}.dW", i, o_, T, True, False, (1.0, 1.0)))
    return out


def operands(rng: DeviceRandom, M: int, N: int, K: int, stds):
    """f32 operands from the generator (A: M x K values, B: K x N values, in their stored order) and their bf16
    roundings on the device."""
    a = rng.normal_(torch.empty(M * K, device="cuda"), stds[0])
    b = rng.normal_(torch.empty(K * N, device="cuda"), stds[1])
    return a, b, a.bfloat16(), b.bfloat16()


def expected_rows(spec: MatmulSpec, left_rows: np.ndarray, right: np.ndarray, r0: int, r1: int) -> np.ndarray:
    """Output rows [r0, r1) of the CPU loop, from op(A)'s rows r0..r1 (`left_rows`: those rows, or for a transposed
    A the matching K x (r1 - r0) block of its stored columns) and the whole right operand."""
    p = spec.product()
    n = r1 - r0
    left_strides = (1, n, 0) if p.left.col_stride != 1 else (spec.inner, 1, 0)
    q = o.product(n, spec.cols, spec.inner, left_strides, (p.right.row_stride, p.right.col_stride, 0), 0)
    out = np.zeros(n * spec.cols, np.float32)
    o.matmul_rows(q, 1, left_rows, right, out, 0, n)
    return out


def left_rows(a, spec: MatmulSpec, r0: int, r1: int) -> np.ndarray:
    """Rows r0..r1 of op(A) as the host needs them (f32), copied from the device operand `a`."""
    M, K = spec.rows, spec.inner
    if spec.product().left.col_stride != 1:   # stored K x M: a column block
        return a.view(K, M)[:, r0:r1].float().contiguous().cpu().numpy().ravel()
    return a[r0 * K:r1 * K].float().cpu().numpy()


def check_product(gpu, rng, name, M, N, K, lt, rt, stds, rows, full_fp32=False):
    spec = MatmulSpec.new(M, N, K)
    if lt:
        spec = spec.left_transposed()
    if rt:
        spec = spec.right_transposed()
    a32, b32, a16, b16 = operands(rng, M, N, K, stds)
    out = torch.empty(M * N, device="cuda")
    gpu.matmul(spec, a16, b16, out)
    assert _ffi.last_path() in _ffi.TENSOR_CORE_PATHS, name
    torch.cuda.synchronize()
    got = out.view(M, N)
    b_r, b_f = b16.float().cpu().numpy(), b32.cpu().numpy()
    for r0, r1 in rows:
        actual = got[r0:r1].cpu().numpy().ravel()
        same_operands = expected_rows(spec, left_rows(a16, spec, r0, r1), b_r, r0, r1)
        err = o.relative_error(same_operands, actual)
        assert err <= 2e-5 * max(1.0, (K / 1024) ** 0.5), (name, r0, err)
    for r0, r1 in ([(0, M)] if full_fp32 else rows):
        fp32_path = expected_rows(spec, left_rows(a32, spec, r0, r1), b_f, r0, r1)
        frob = o.relative_frobenius(fp32_path, got[r0:r1].cpu().numpy().ravel())
        assert frob <= 1e-2, (name, r0, frob)
    del a32, b32, a16, b16, out, got
    gpu.device_status()


@pytest.mark.parametrize("cfg", [1, 2])
def test_every_block_gemm_in_full_tensors(gpu, cfg):
    T, w = CONFIGS[cfg]
    rng = DeviceRandom(gpu, 0)
    for case in block_gemms(T, w):
        M = case[1]
        check_product(gpu, rng, *case, rows=[(0, 32), (M // 2 - 16, M // 2 + 16), (M - 32, M)], full_fp32=True)


def test_config3_sampled_rows_of_every_gemm_shape_and_the_head(gpu):
    T, w = CONFIGS[3]
    rng = DeviceRandom(gpu, 0)
    cases = block_gemms(T, w) + [
        ("head.fwd", T, 16 * 1024, w, False, False, (1.0, 1.0 / np.sqrt(w))),
        ("head.dX", T, w, 16 * 1024, False, True, (1.0, 1.0 / np.sqrt(w))),
        ("head.dW", w, 16 * 1024, T, True, False, (1.0, 1.0)),
    ]
    for name, M, N, K, lt, rt, stds in cases:
        # First, middle and last full rows; fewer when a row costs a whole K = 65,536 reduction per column.
        n = 4 if K >= T else 16
        rows = [(0, n), (M // 2 - n // 2, M // 2 + n // 2), (M - n, M)]
        check_product(gpu, rng, name, M, N, K, lt, rt, stds, rows=rows)
        torch.cuda.empty_cache()


@pytest.mark.parametrize("deterministic", [False, True])
def test_config3_weight_gradients_in_full_against_float64(gpu, deterministic):
    # Every element of config 3's weight-gradient products (K = 65,536 tokens, split along K up to 19 ways) and the
    # head's, accumulated into an initial gradient as the step does (linear.rs:55-57), against a float64 product of
    # the same bf16 operands on the device: what remains is the f32 accumulation of the tensor core and of the
    # split-K sums, so a lost or doubled K slice at any split boundary shows at once (a lost 16-row slice alone moves
    # the result by ~1.5e-2). Bound: the file's summation-order bar, 2e-5 * sqrt(K/1024) = 1.6e-4 as a relative
    # Frobenius error (3.5e-5 measured on expand.dW).
    T, w = CONFIGS[3]
    rng = DeviceRandom(gpu, 1)
    shapes = [("qkv.dW", w, 3 * w), ("output.dW", w, w), ("expand.dW", w, 4 * w), ("project.dW", 4 * w, w),
              ("head.dW", w, 16 * 1024)]
    for name, M, N in shapes:
        x = rng.normal_(torch.empty(T, M, device="cuda")).bfloat16()
        dy = rng.normal_(torch.empty(T, N, device="cuda")).bfloat16()
        initial = rng.normal_(torch.empty(M, N, device="cuda"), 100.0)
        dw = initial.clone()
        gpu.gemm(MatmulSpec.new(M, N, T).left_transposed().accumulate(), x, dy, dw, deterministic=deterministic)
        assert _ffi.last_path() in _ffi.TENSOR_CORE_PATHS, name
        exact = initial.double() + x.double().t() @ dy.double()
        err = (torch.linalg.vector_norm(dw.double() - exact) / torch.linalg.vector_norm(exact)).item()
        assert err <= 2e-5 * (T / 1024) ** 0.5, (name, err)
        del x, dy, initial, dw, exact
        torch.cuda.empty_cache()
    gpu.device_status()
