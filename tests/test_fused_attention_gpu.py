"""Fused causal attention forward (snb_causal_attention_forward) against the oracle composition of the reference's
QK^T product, causal_softmax and P.V product (crates/staleynet-model/src/layers/attention.rs:206-213,
crates/staleynet-cuda/src/reference.rs:100-120) on the same bf16 inputs. The fused kernel rounds the unnormalised
probabilities to bf16 for its P.V product, so the bound is the bf16 one (relative Frobenius <= 1e-2)."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import oracle as o  # noqa: E402
from staleynet_b200 import _ffi  # noqa: E402
from staleynet_b200.matmul import Gpu  # noqa: E402

pytestmark = pytest.mark.gpu


def oracle_attention(q, k, v, offset, scale):
    """q [Sq, d], k/v [Sk, d] f32 -> (out [Sq, d], lse [Sq])."""
    Sq, d = q.shape
    Sk = k.shape[0]
    scores = np.zeros(Sq * Sk, np.float32)
    p = o.product(Sq, Sk, d, o.storage_strides(False, Sq, d, 0), o.storage_strides(True, d, Sk, 0), 0)
    o.matmul_rows(p, 1, np.ascontiguousarray(q).ravel(), np.ascontiguousarray(k).ravel(), scores, 0, Sq)
    raw = scores.reshape(Sq, Sk).astype(np.float64)
    o.causal_softmax(scores, Sq, Sk, scale, offset)
    out = np.zeros(Sq * d, np.float32)
    p2 = o.product(Sq, d, Sk, o.storage_strides(False, Sq, Sk, 0), o.storage_strides(False, Sk, d, 0), 0)
    o.matmul_rows(p2, 1, scores, np.ascontiguousarray(v).ravel(), out, 0, Sq)
    lse = np.empty(Sq)
    for i in range(Sq):
        vis = min(i + offset + 1, Sk)
        x = raw[i, :vis] * scale
        mx = x.max()
        lse[i] = mx + np.log(np.exp(x - mx).sum())
    return out.reshape(Sq, d), lse


@pytest.mark.parametrize("count,sq,sk,offset,out_type", [
    (2, 200, 200, 0, "f32"), (3, 384, 384, 0, "bf16"), (2, 130, 300, 170, "f32"), (4, 1, 257, 256, "f32"),
    (1, 513, 513, 0, "f32"), (2, 256, 256, 3, "bf16")])
def test_fused_attention_matches_the_oracle(count, sq, sk, offset, out_type):
    torch.manual_seed(0)
    gpu = Gpu(0)
    q = torch.randn(count, sq, 64, device="cuda").bfloat16()
    k = torch.randn(count, sk, 64, device="cuda").bfloat16()
    v = torch.randn(count, sk, 64, device="cuda").bfloat16()
    dt = torch.bfloat16 if out_type == "bf16" else torch.float32
    out = torch.full((count, sq, 64), 7.0, device="cuda", dtype=dt)
    lse = torch.zeros(count, sq, device="cuda")
    scale = 0.125
    gpu.causal_attention_forward(q, k, v, out, scale, offset, lse)
    torch.cuda.synchronize()
    assert _ffi.load().snb_device_status() == _ffi.OK
    for b in range(count):
        e_out, e_lse = oracle_attention(q[b].float().cpu().numpy(), k[b].float().cpu().numpy(),
                                        v[b].float().cpu().numpy(), offset, scale)
        got = out[b].float().cpu().numpy()
        assert o.relative_frobenius(e_out, got) < 1e-2, f"matrix {b}"
        assert o.relative_error(e_out, got) < 3e-2, f"matrix {b}"
        assert np.max(np.abs(lse[b].cpu().numpy() - e_lse)) < 1e-3, f"matrix {b} lse"


def test_fused_attention_equals_the_materialised_path_at_baseline_config4():
    """BASELINE config 4 (batch 8, 12 heads of 64, sequence 3072): the fused forward agrees with the materialised
    QK^T -> causal softmax -> P.V path of staleynet_b200.attention on every head."""
    from staleynet_b200.attention import AttentionProducts, AttentionShape

    att = AttentionProducts(AttentionShape(), torch.device("cuda", 0), seed=5)
    h = torch.cuda.current_stream().cuda_stream
    att.forward(h)
    s = att.shape
    out = torch.empty(s.count, s.time, 64, device="cuda")
    Gpu(0).causal_attention_forward(att.q.view(s.count, s.time, 64), att.k.view(s.count, s.time, 64),
                                    att.v.view(s.count, s.time, 64), out, att.scale, 0)
    torch.cuda.synchronize()
    ref = att.ctx.view(s.count, s.time, 64)
    err = (torch.linalg.vector_norm(out - ref) / torch.linalg.vector_norm(ref)).item()
    assert err < 1e-2
    assert _ffi.load().snb_device_status() == _ffi.OK


def oracle_attention_backward(q, k, v, do, offset, scale):
    """The reference's attention backward (attention.rs:220-267) on f32 inputs: P by the oracle causal_softmax,
    dS by the oracle softmax_backward, the products in float64."""
    Sq, Sk = q.shape[0], k.shape[0]
    scores = (q.astype(np.float64) @ k.astype(np.float64).T).astype(np.float32).ravel()
    o.causal_softmax(scores, Sq, Sk, scale, offset)
    P = scores.reshape(Sq, Sk)
    dS = (do.astype(np.float64) @ v.astype(np.float64).T).astype(np.float32).ravel()
    o.softmax_backward(np.ascontiguousarray(P.ravel()), dS, Sk)
    dS = dS.reshape(Sq, Sk).astype(np.float64)
    dq = scale * dS @ k.astype(np.float64)
    dk = scale * dS.T @ q.astype(np.float64)
    dv = P.astype(np.float64).T @ do.astype(np.float64)
    return dq, dk, dv


@pytest.mark.parametrize("count,sq,sk,offset,out_type", [
    (2, 200, 200, 0, "f32"), (3, 384, 384, 0, "bf16"), (2, 130, 300, 170, "f32"), (4, 1, 257, 256, "f32"),
    (1, 513, 513, 0, "f32"), (2, 256, 256, 3, "bf16"), (1, 100, 300, 0, "f32")])
def test_fused_attention_backward_matches_the_oracle(count, sq, sk, offset, out_type):
    """Ragged sizes, query offsets, and (last case) key tiles that no query sees, whose dK and dV must be zero."""
    torch.manual_seed(1)
    gpu = Gpu(0)
    q = torch.randn(count, sq, 64, device="cuda").bfloat16()
    k = torch.randn(count, sk, 64, device="cuda").bfloat16()
    v = torch.randn(count, sk, 64, device="cuda").bfloat16()
    do = torch.randn(count, sq, 64, device="cuda").bfloat16()
    dt = torch.bfloat16 if out_type == "bf16" else torch.float32
    out = torch.empty(count, sq, 64, device="cuda", dtype=dt)
    lse = torch.empty(count, sq, device="cuda")
    scale = 0.125
    gpu.causal_attention_forward(q, k, v, out, scale, offset, lse)
    dq = torch.full((count, sq, 64), 5.0, device="cuda")
    dk = torch.full((count, sk, 64), 5.0, device="cuda")
    dv = torch.full((count, sk, 64), 5.0, device="cuda")
    gpu.causal_attention_backward(q, k, v, out, do, lse, dq, dk, dv, scale, offset)
    torch.cuda.synchronize()
    assert _ffi.load().snb_device_status() == _ffi.OK
    for b in range(count):
        e_dq, e_dk, e_dv = oracle_attention_backward(q[b].float().cpu().numpy(), k[b].float().cpu().numpy(),
                                                     v[b].float().cpu().numpy(), do[b].float().cpu().numpy(),
                                                     offset, scale)
        for name, e, g in (("dq", e_dq, dq[b]), ("dk", e_dk, dk[b]), ("dv", e_dv, dv[b])):
            got = g.cpu().numpy()
            assert o.relative_frobenius(e, got) < 1e-2, f"matrix {b} {name}"
        seen = min(sk, sq - 1 + offset + 1)   # keys at or past `seen` are visible to no query
        assert np.all(dk[b, seen:].cpu().numpy() == 0) and np.all(dv[b, seen:].cpu().numpy() == 0)


def test_fused_attention_backward_equals_the_materialised_path_at_baseline_config4():
    """the fused backward agrees with the materialised dP, dV, softmax-backward, dQ, dK products of
    staleynet_b200.attention on every head."""
    from staleynet_b200.attention import AttentionProducts, AttentionShape

    att = AttentionProducts(AttentionShape(), torch.device("cuda", 0), seed=7)
    h = torch.cuda.current_stream().cuda_stream
    att.forward(h)
    att.backward(h)
    s = att.shape
    view = lambda t: t.view(s.count, s.time, 64)  # noqa: E731
    gpu = Gpu(0)
    out = torch.empty(s.count, s.time, 64, device="cuda")
    lse = torch.empty(s.count, s.time, device="cuda")
    gpu.causal_attention_forward(view(att.q), view(att.k), view(att.v), out, att.scale, 0, lse)
    dq, dk, dv = (torch.empty(s.count, s.time, 64, device="cuda") for _ in range(3))
    gpu.causal_attention_backward(view(att.q), view(att.k), view(att.v), out, view(att.d_out), lse, dq, dk, dv,
                                  att.scale, 0)
    torch.cuda.synchronize()
    assert _ffi.load().snb_device_status() == _ffi.OK
    for name, got, ref in (("dq", dq, att.dq), ("dk", dk, att.dk), ("dv", dv, att.dv)):
        ref = view(ref)
        err = (torch.linalg.vector_norm(got - ref) / torch.linalg.vector_norm(ref)).item()
        assert err < 1e-2, name
