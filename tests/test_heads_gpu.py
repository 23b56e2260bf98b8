"""Attention head layouts on the GPU: the reference's split_heads / merge_heads permutes (crates/staleynet-cuda/src/
kernels/attention.rs:112-138) through snb_split_heads / snb_merge_heads / snb_permute_heads, the same permutes fused
into the products around attention (snb_gemm left_heads / output_heads), and `CausalSelfAttention`'s forward and
backward (crates/staleynet-model/src/layers/attention.rs:188-267) run from packed activations to packed gradients on
the C ABI alone, against the oracle composition."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import oracle as o  # noqa: E402
from staleynet_b200 import _ffi  # noqa: E402
from staleynet_b200._ffi import HeadLayout  # noqa: E402
from staleynet_b200.attention import CausalSelfAttentionLayer, LayerShape  # noqa: E402
from staleynet_b200.matmul import Gpu, MatmulKernel, MatmulSpec, SnbError  # noqa: E402

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def gpu():
    return Gpu(0)


def _rel(expected, actual):
    e = np.asarray(expected, np.float64)
    return float(np.linalg.norm(np.asarray(actual, np.float64) - e) / np.linalg.norm(e))


def test_split_and_merge_heads_follow_the_layout_formula(gpu):
    # The reference's split_and_merge_heads_follow_the_layout_formula (crates/staleynet-cuda/tests/
    # kernels_match_reference.rs:199-231), bit for bit: odd head_dim, a packed row wider than the heads, a cache.
    L = HeadLayout.dense(2, 5, 3, 4, 3 * 12 + 2, 13).in_cache(9, 2)
    packed = o.lcg_values(L.batch * L.time * L.width, 12)
    head_major = torch.zeros(L.batch * L.heads * L.time_capacity * L.head_dim, device="cuda")
    gpu.split_heads(torch.from_numpy(packed).cuda(), head_major, L)
    expected = np.zeros(head_major.numel(), np.float32)
    o.split_heads(packed, expected, L)
    assert np.array_equal(head_major.cpu().numpy(), expected)
    merged = torch.zeros(packed.size, device="cuda")
    gpu.merge_heads(head_major, merged, L)
    back = np.zeros_like(packed)
    o.merge_heads(expected, back, L)
    assert np.array_equal(merged.cpu().numpy(), back)


@pytest.mark.parametrize("src_dtype,dst_dtype", [(torch.float32, torch.float32), (torch.float32, torch.bfloat16),
                                                 (torch.bfloat16, torch.bfloat16), (torch.bfloat16, torch.float32)])
@pytest.mark.parametrize("direction", [_ffi.HEADS_SPLIT, _ffi.HEADS_MERGE])
def test_permutes_of_model_layouts_in_both_directions_and_types(gpu, src_dtype, dst_dtype, direction):
    # The model's layouts (12 heads of 64 in a fused 3 x 768 row, keys at column 768) move 16 bytes per thread; a
    # cache offset and capacity as in forward_cached (attention.rs:292-299).
    L = HeadLayout.dense(3, 96, 12, 64, 3 * 768, 768).in_cache(160, 40)
    n_packed = L.batch * L.time * L.width
    n_heads = L.batch * L.heads * L.time_capacity * L.head_dim
    src_np = o.lcg_values(n_packed if direction == _ffi.HEADS_SPLIT else n_heads, 3)
    src = torch.from_numpy(src_np).cuda().to(src_dtype)
    dst = torch.full((n_heads if direction == _ffi.HEADS_SPLIT else n_packed,), -5.0, device="cuda", dtype=dst_dtype)
    gpu.permute_heads(direction, src, dst, L)
    # Expected: the oracle's permute of the source values, converted once to the destination type.
    src_vals = src.float().cpu().numpy()
    exp = dst.float().cpu().numpy().copy() * 0 - 5.0
    if direction == _ffi.HEADS_SPLIT:
        o.split_heads(src_vals, exp, L)
    else:
        o.merge_heads(src_vals, exp, L)
    expected = torch.from_numpy(exp).to(dst_dtype).float().numpy()
    assert np.array_equal(dst.float().cpu().numpy(), expected)


def _qkv_case(T, w, dtype):
    g = torch.Generator(device="cuda").manual_seed(7)
    x = torch.randn(T, w, device="cuda", generator=g).to(dtype)
    wq = (torch.randn(w, 3 * w, device="cuda", generator=g) / w ** 0.5).to(dtype)
    b = torch.randn(3 * w, device="cuda", generator=g)
    return x, wq, b


@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float32])
def test_gemm_written_head_major_equals_the_packed_product_then_split(gpu, out_dtype):
    # The fused QKV projection: 2 sequences x 256 steps, 4 heads of 64, written into a cache of 320 steps from step
    # 32 (the rest of the cache keeps its contents).
    B, S, H, d = 2, 256, 4, 64
    w, T = H * d, B * S
    x, wq, b = _qkv_case(T, w, torch.bfloat16)
    spec = MatmulSpec.new(T, 3 * w, w)
    packed = torch.empty(T, 3 * w, device="cuda", dtype=out_dtype)
    gpu.gemm(spec, x, wq, packed, bias=b)
    L = HeadLayout.dense(B, S, H, d, 3 * w, 0).in_cache(320, 32)
    fused = torch.full((3, B * H, 320, d), 3.0, device="cuda", dtype=out_dtype)
    gpu.gemm(spec, x, wq, fused, bias=b, output_heads=L)
    assert _ffi.last_path() in _ffi.TENSOR_CORE_PATHS
    expected = torch.full_like(fused, 3.0)
    for p in range(3):
        gpu.split_heads(packed, expected[p], HeadLayout.dense(B, S, H, d, 3 * w, p * w).in_cache(320, 32))
    torch.cuda.synchronize()
    assert torch.equal(fused, expected)


@pytest.mark.parametrize("kernel", [MatmulKernel.BF16_TENSOR_CORE, MatmulKernel.TENSOR_CORE])
def test_gemm_reading_head_major_equals_the_packed_product(gpu, kernel):
    # The output projection reads the attention context head-major (RowMajor: tokens x features) and its weight
    # gradient reads it transposed (features x tokens); both equal the products on the packed context bit for bit
    # (same operand values, same summation order; the dW runs deterministic).
    B, S, H, d = 2, 256, 3, 64
    w, T = H * d, B * S
    dtype = torch.bfloat16 if kernel is MatmulKernel.BF16_TENSOR_CORE else torch.float32
    gpu.matmul_kernel = kernel
    g = torch.Generator(device="cuda").manual_seed(9)
    heads = torch.randn(B * H, S, d, device="cuda", generator=g).to(dtype)
    packed = torch.empty(T, w, device="cuda", dtype=dtype)
    L = HeadLayout.dense(B, S, H, d, w, 0)
    gpu.merge_heads(heads, packed, L)
    wo = torch.randn(w, w, device="cuda", generator=g).to(dtype)
    dy = torch.randn(T, w, device="cuda", generator=g).to(dtype)
    y_ref, y = (torch.empty(T, w, device="cuda") for _ in range(2))
    gpu.gemm(MatmulSpec.new(T, w, w), packed, wo, y_ref)
    gpu.gemm(MatmulSpec.new(T, w, w), heads, wo, y, left_heads=L)
    assert _ffi.last_path() in _ffi.TENSOR_CORE_PATHS
    dw_spec = MatmulSpec.new(w, w, T).left_transposed().accumulate()
    dw_ref, dw = (torch.ones(w, w, device="cuda") for _ in range(2))
    gpu.gemm(dw_spec, packed, dy, dw_ref, deterministic=True)
    gpu.gemm(dw_spec, heads, dy, dw, left_heads=L, deterministic=True)
    torch.cuda.synchronize()
    assert torch.equal(y, y_ref)
    assert torch.equal(dw, dw_ref)


def test_gemm_head_layouts_that_no_kernel_can_fuse_are_refused(gpu):
    # 100 steps per sequence: a 32-row output box would straddle two sequences.
    B, S, H, d = 2, 100, 2, 64
    w, T = H * d, B * S
    x, wq, b = _qkv_case(T, w, torch.bfloat16)
    out = torch.empty(3, B * H, S, d, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(SnbError) as e:
        gpu.gemm(MatmulSpec.new(T, 3 * w, w), x, wq, out, output_heads=HeadLayout.dense(B, S, H, d, 3 * w, 0))
    assert e.value.code == _ffi.ERR_UNSUPPORTED


def _layer_oracle(layer, x, dy):
    """CausalSelfAttention::forward / backward (attention.rs:188-267) restated on the CPU: float64 products, the
    oracle's causal_softmax and softmax_backward (reference.rs:100-137), the oracle's head permutes, and bf16
    rounding where the GPU layer stores bf16 tensors (qkv, the context, its gradient, the qkv gradient)."""
    s = layer.shape
    B, S, H, d, w, T = s.batch, s.time, s.heads, s.head_dim, s.width, s.tokens
    f = lambda t: t.float().cpu().numpy().astype(np.float64)  # noqa: E731
    bf = lambda a: torch.from_numpy(np.asarray(a, np.float32)).bfloat16().float().numpy().astype(np.float64)  # noqa
    X, Wq, bq, Wo, bo, dY = f(x), f(layer.w_qkv), f(layer.b_qkv), f(layer.w_o), f(layer.b_o), f(dy)
    qkv = bf(X @ Wq + bq).reshape(-1)
    n = B * H * S * d
    heads = []
    for p in range(3):
        hm = np.zeros(n)
        o.split_heads(qkv, hm, HeadLayout.dense(B, S, H, d, 3 * w, p * w))
        heads.append(hm.reshape(B * H, S, d))
    q, k, v = heads
    scores = np.einsum("nqd,nkd->nqk", q, k).astype(np.float32).reshape(-1)
    o.causal_softmax(scores, S, S, layer.scale, 0)
    P = scores.reshape(B * H, S, S).astype(np.float64)
    ctx_h = bf(np.einsum("nqk,nkd->nqd", P, v))
    ctx = np.zeros(T * w)
    o.merge_heads(ctx_h.reshape(-1), ctx, HeadLayout.dense(B, S, H, d, w, 0))
    ctx = ctx.reshape(T, w)
    y = ctx @ Wo + bo
    g_wo = ctx.T @ dY
    d_ctx = bf(dY @ Wo.T).reshape(-1)
    do = np.zeros(n)
    o.split_heads(d_ctx, do, HeadLayout.dense(B, S, H, d, w, 0))
    do = do.reshape(B * H, S, d)
    dP = np.einsum("nqd,nkd->nqk", do, v).astype(np.float32).reshape(-1)
    dV = np.einsum("nqk,nqd->nkd", P, do)
    Pf = P.astype(np.float32).reshape(-1)
    o.softmax_backward(Pf, dP, S)
    dS = dP.reshape(B * H, S, S).astype(np.float64)
    dQ = layer.scale * np.einsum("nqk,nkd->nqd", dS, k)
    dK = layer.scale * np.einsum("nqk,nqd->nkd", dS, q)
    d_qkv = np.zeros(T * 3 * w)
    for p, gh in enumerate((dQ, dK, dV)):
        o.merge_heads(gh.reshape(-1), d_qkv, HeadLayout.dense(B, S, H, d, 3 * w, p * w))
    d_qkv = bf(d_qkv).reshape(T, 3 * w)
    g_wqkv = X.T @ d_qkv
    dx = d_qkv @ Wq.T
    return y, dx, g_wqkv, g_wo


def _run_layer(layer, x, dy):
    s = layer.shape
    y = torch.empty(s.tokens, s.width, device="cuda", dtype=torch.bfloat16)
    dx = torch.empty_like(y)
    layer.forward(x, y)
    layer.backward(x, dy, dx)
    torch.cuda.synchronize()
    return y, dx


def test_attention_layer_on_the_c_abi_matches_the_oracle_composition():
    shape = LayerShape(batch=2, time=256, heads=2, head_dim=64)
    layer = CausalSelfAttentionLayer(shape, torch.device("cuda", 0), seed=4)
    g = torch.Generator(device="cuda").manual_seed(11)
    x = torch.randn(shape.tokens, shape.width, device="cuda", generator=g).bfloat16()
    dy = torch.randn(shape.tokens, shape.width, device="cuda", generator=g).bfloat16()
    y, dx = _run_layer(layer, x, dy)
    ey, edx, eg_wqkv, eg_wo = _layer_oracle(layer, x, dy)
    # bf16 operands throughout (P and dS are rounded to bf16 inside the fused attention kernels): BASELINE's bf16
    # tolerance, relative Frobenius <= 1e-2.
    assert _rel(ey, y.float().cpu().numpy()) < 1e-2
    assert _rel(edx, dx.float().cpu().numpy()) < 1e-2
    assert _rel(eg_wqkv, layer.g_wqkv.cpu().numpy()) < 1e-2
    assert _rel(eg_wo, layer.g_wo.cpu().numpy()) < 1e-2


def test_fused_permutes_give_the_unfused_layer_bit_for_bit():
    # The permutes fused into the products move the same values as the separate permute kernels, so the two layers
    # agree exactly up to the attention backward (weight gradients deterministic); dq's reductions are unordered, so
    # dx and dWqkv, which depend on it through bf16 rounding, are compared within tolerance.
    shape = LayerShape(batch=2, time=384, heads=3, head_dim=64)
    dev = torch.device("cuda", 0)
    fused = CausalSelfAttentionLayer(shape, dev, seed=5, fused_permutes=True, deterministic=True)
    plain = CausalSelfAttentionLayer(shape, dev, seed=5, fused_permutes=False, deterministic=True)
    g = torch.Generator(device="cuda").manual_seed(12)
    x = torch.randn(shape.tokens, shape.width, device="cuda", generator=g).bfloat16()
    dy = torch.randn(shape.tokens, shape.width, device="cuda", generator=g).bfloat16()
    yf, dxf = _run_layer(fused, x, dy)
    yp, dxp = _run_layer(plain, x, dy)
    assert torch.equal(yf, yp)
    assert torch.equal(fused.g_wo, plain.g_wo)
    assert torch.equal(fused.do_heads, plain.do_heads)
    assert _rel(dxp.float().cpu().numpy(), dxf.float().cpu().numpy()) < 1e-2
    assert _rel(plain.g_wqkv.cpu().numpy(), fused.g_wqkv.cpu().numpy()) < 1e-3
