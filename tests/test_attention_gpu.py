"""The batched attention products (crates/staleynet-model/src/layers/attention.rs:188-267) with their causal hints,
against the CPU oracle composed in the reference's order: QK^T, causal softmax, P.V and the backward products with
softmax_backward between them. The GPU path runs bf16 tensor-core products on bf16 copies of P and dS, so the oracle
composition rounds P and dS to bf16 at the same points; masked score entries are unspecified (never read)."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import oracle as o  # noqa: E402
from staleynet_b200 import _ffi  # noqa: E402
from staleynet_b200.attention import AttentionProducts, AttentionShape  # noqa: E402

pytestmark = pytest.mark.gpu


def oracle_head(q, k, v, dout, S, d, offset, scale):
    """One matrix of the batch through the oracle; f32 numpy arrays [S, d]."""
    def mm(a, b, M, N, K, lt=False, rt=False, sc=1.0):
        out = np.zeros(M * N, np.float32)
        p = o.product(M, N, K, o.storage_strides(lt, M, K, 0), o.storage_strides(rt, K, N, 0), 0, sc, False)
        o.matmul_rows(p, 1, np.ascontiguousarray(a).ravel(), np.ascontiguousarray(b).ravel(), out, 0, M)
        return out.reshape(M, N)

    scores = mm(q, k, S, S, d, rt=True)
    p = scores.copy().ravel()
    o.causal_softmax(p, S, S, scale, offset)
    p = p.reshape(S, S)
    p16, _ = o.round_bf16(p)
    ctx = mm(p16, v, S, d, S)
    dp = mm(dout, v, S, S, d, rt=True)
    dv = mm(p16, dout, S, d, S, lt=True)
    ds = dp.copy().ravel()
    o.softmax_backward(p.ravel().copy(), ds, S)
    ds = ds.reshape(S, S)
    ds16, _ = o.round_bf16(ds)
    dq = mm(ds16, k, S, d, S, sc=scale)
    dk = mm(ds16, q, S, d, S, lt=True, sc=scale)
    return scores, p, ctx, dv, ds, dq, dk


def check_heads(att, heads):
    s = att.shape
    S, d = s.time, s.head_dim
    as_np = lambda t: t.float().cpu().numpy()  # noqa: E731
    q, k, v, dout = (as_np(t).reshape(s.count, S, d) for t in (att.q, att.k, att.v, att.d_out))
    scores = as_np(att.scores).reshape(s.count, S, S)
    ctx, dq, dk, dv = (as_np(t).reshape(s.count, S, d) for t in (att.ctx, att.dq, att.dk, att.dv))
    ds = as_np(att.d_scores).reshape(s.count, S, S)
    visible = np.tril(np.ones((S, S), bool), k=s.query_offset)
    for h in heads:
        e_scores, e_p, e_ctx, e_dv, e_ds, e_dq, e_dk = oracle_head(q[h], k[h], v[h], dout[h], S, d, s.query_offset,
                                                                    att.scale)
        assert o.relative_error(e_p, scores[h]) < 1e-4, "probabilities"
        assert np.all(scores[h][~visible] == 0), "masked probabilities must be 0"
        assert np.all(ds[h][~visible] == 0), "masked score gradients must be 0"
        for name, e, a in (("ctx", e_ctx, ctx[h]), ("dV", e_dv, dv[h]), ("dS", e_ds, ds[h]), ("dQ", e_dq, dq[h]),
                           ("dK", e_dk, dk[h])):
            err = o.relative_frobenius(e, a)
            assert err < 5e-3, f"head {h} {name}: relative Frobenius {err}"
        del e_scores


@pytest.mark.parametrize("S,offset", [(200, 0), (200, 7), (384, 0)])
def test_attention_products_with_causal_hints_match_the_oracle(S, offset):
    torch.cuda.set_device(0)
    att = AttentionProducts(AttentionShape(batch=2, heads=2, time=S, head_dim=64, query_offset=offset),
                            torch.device("cuda", 0), seed=3)
    h = torch.cuda.current_stream().cuda_stream
    att.forward(h)
    att.backward(h)
    torch.cuda.synchronize()
    check_heads(att, range(att.shape.count))
    assert _ffi.load().snb_device_status() == _ffi.OK


def test_causal_output_skip_leaves_masked_tiles_untouched():
    """SKIP_MASKED_OUTPUT computes every visible score and no tile that is entirely masked."""
    from staleynet_b200.matmul import BatchStrides, Gpu, MatmulSpec

    gpu = Gpu(0)
    S, d, n = 520, 64, 2
    q = torch.randn(n * S * d, device="cuda").bfloat16()
    k = torch.randn(n * S * d, device="cuda").bfloat16()
    out = torch.full((n * S * S,), 12345.0, device="cuda")
    spec = MatmulSpec.new(S, S, d).right_transposed().batched(BatchStrides(n, S * d, S * d, S * S))
    gpu.gemm(spec, q, k, out, causal=_ffi.CAUSAL_SKIP_MASKED_OUTPUT)
    ref = torch.bmm(q.float().view(n, S, d), k.float().view(n, S, d).transpose(1, 2))
    got = out.view(n, S, S)
    vis = torch.tril(torch.ones(S, S, dtype=torch.bool, device="cuda"))
    assert torch.allclose(got[:, vis], ref[:, vis], rtol=1e-3, atol=1e-2)
    rows = torch.arange(S, device="cuda").view(S, 1)
    cols = torch.arange(S, device="cuda").view(1, S)
    whole_tile_masked = (cols // 256) * 256 > (rows // 128) * 128 + 127
    assert torch.all(got[:, whole_tile_masked] == 12345.0)


def test_baseline_config4_attention_at_full_size_on_sampled_heads():
    """BASELINE config 4 (batch 8, 12 heads of 64, sequence 3072) end to end on the GPU; two heads checked in full
    against the oracle (a size-independent property: every head is computed the same way)."""
    torch.cuda.set_device(0)
    att = AttentionProducts(AttentionShape(), torch.device("cuda", 0), seed=0)
    h = torch.cuda.current_stream().cuda_stream
    att.forward(h)
    att.backward(h)
    torch.cuda.synchronize()
    check_heads(att, [0, att.shape.count - 1])
    assert _ffi.load().snb_device_status() == _ffi.OK
