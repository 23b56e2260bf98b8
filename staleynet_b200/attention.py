"""The batched attention products of `CausalSelfAttention` (crates/staleynet-model/src/layers/attention.rs:188-267)
through the C ABI, on head-major tensors [batch*heads, time, head_dim], with the fp32 causal softmax between them:

  forward   scores = Q·Kᵀ                     MatmulSpec(S, S, d).right_transposed()   (attention.rs:206-209)
            P      = causal_softmax(scores)                                            (attention.rs:210)
            ctx    = P·V                      MatmulSpec(S, d, S)                      (attention.rs:212-213)
  backward  dP     = dO·Vᵀ                                                              (attention.rs:239-242)
            dV     = Pᵀ·dO                    .left_transposed()                        (attention.rs:244-247)
            dS     = softmax_backward(P, dP)                                            (attention.rs:249)
            dQ     = s·dS·K                   .scaled(s)                                (attention.rs:251-254)
            dK     = s·dSᵀ·Q                  .left_transposed().scaled(s)              (attention.rs:256-260)

Q, K, V, dO are bf16; scores, P, dP and dS are f32 as in the reference, and the softmax kernels also write bf16
copies of P and dS so that every product runs on bf16 tensor cores. Each product carries its causal hint
(SNB_CAUSAL_*): masked score tiles are not computed, and products over P or dS stop or start their sum where the
causal mask makes the operand zero. ctx, dQ, dK and dV are f32.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

from . import _ffi
from .matmul import BatchStrides, DeviceRandom, Gpu, MatmulSpec, check


@dataclass(frozen=True)
class AttentionShape:
    """batch 8, 12 heads of 64, sequence 3072."""

    batch: int = 8
    heads: int = 12
    time: int = 3072
    head_dim: int = 64
    query_offset: int = 0

    @property
    def count(self) -> int:
        return self.batch * self.heads


def causal_pairs(s: AttentionShape) -> int:
    """Visible (query, key) pairs of one matrix: sum over q of min(q + offset + 1, time)."""
    S, o = s.time, s.query_offset
    return sum(min(q + o + 1, S) for q in range(S))


def product_flops(s: AttentionShape, causal: bool = True) -> float:
    """FLOPs of the six products: 2*d per visible (causal) or every (dense) query-key pair, per product."""
    pairs = causal_pairs(s) if causal else s.time * s.time
    return 6 * 2.0 * s.head_dim * pairs * s.count


def algorithmic_bytes(s: AttentionShape) -> float:
    """Bytes the forward + backward must move at the types above: every operand read once, every output written
    once; score-shaped f32 tensors are written in full by the softmax kernels (masked entries become 0, the
    reference's contract) and read over their visible part only."""
    S, d, n = s.time, s.head_dim, s.count
    vis = causal_pairs(s)
    head = S * d
    fwd = (2 * head * 2 + vis * 4           # Q, K read; visible scores written
           + vis * 4 + S * S * (4 + 2)      # softmax: visible read, full f32 + bf16 written
           + vis * 2 + head * 2 + head * 4)  # P.V: bf16 P visible, V, ctx f32
    bwd = (2 * head * 2 + vis * 4           # dO, V read; visible dP written
           + vis * 2 + head * 2 + head * 4  # dV = P^T dO
           + 2 * vis * 4 + S * S * (4 + 2)  # softmax backward: P, dP visible read; dS f32 + bf16 written
           + 2 * (vis * 2 + head * 2 + head * 4))  # dQ, dK
    return float(n) * (fwd + bwd)


class AttentionProducts:
    """Device tensors and pre-built C-ABI arguments for the six products of one attention layer call."""

    def __init__(self, shape: AttentionShape, device, seed: int = 0):
        import torch

        s = shape
        self.shape = s
        self.lib = _ffi.load()
        n, S, d = s.count, s.time, s.head_dim
        # Q, K, V and dO from the reference's generator (Random::new(seed), random.rs:27-70), drawn on the device.
        rng = DeviceRandom(Gpu(device.index if device.index is not None else 0), seed)

        def normal(numel):
            return rng.normal_(torch.empty(numel, device=device, dtype=torch.bfloat16))

        bf16, f32 = torch.bfloat16, torch.float32
        self.q, self.k, self.v, self.d_out = (normal(n * S * d) for _ in range(4))
        self.scores = torch.empty(n * S * S, device=device, dtype=f32)      # scores, then P (in place)
        self.p16 = torch.empty(n * S * S, device=device, dtype=bf16)
        self.ctx = torch.empty(n * S * d, device=device, dtype=f32)
        self.d_scores = torch.empty(n * S * S, device=device, dtype=f32)    # dP, then dS (in place)
        self.ds16 = torch.empty(n * S * S, device=device, dtype=bf16)
        self.dq = torch.empty(n * S * d, device=device, dtype=f32)
        self.dk = torch.empty(n * S * d, device=device, dtype=f32)
        self.dv = torch.empty(n * S * d, device=device, dtype=f32)
        self.scale = 1.0 / (d ** 0.5)

        head, score = S * d, S * S
        per_head = lambda left, right, out: BatchStrides(count=n, left=left, right=right, output=out)  # noqa: E731
        C = _ffi
        self.args = {
            "scores": self._args(MatmulSpec.new(S, S, d).right_transposed().batched(per_head(head, head, score)),
                                 self.q, self.k, self.scores, C.CAUSAL_SKIP_MASKED_OUTPUT),
            "ctx": self._args(MatmulSpec.new(S, d, S).batched(per_head(score, head, head)),
                              self.p16, self.v, self.ctx, C.CAUSAL_LEFT_MASKED),
            "dP": self._args(MatmulSpec.new(S, S, d).right_transposed().batched(per_head(head, head, score)),
                             self.d_out, self.v, self.d_scores, C.CAUSAL_SKIP_MASKED_OUTPUT),
            "dV": self._args(MatmulSpec.new(S, d, S).left_transposed().batched(per_head(score, head, head)),
                             self.p16, self.d_out, self.dv, C.CAUSAL_LEFT_T_MASKED),
            "dQ": self._args(MatmulSpec.new(S, d, S).scaled(self.scale).batched(per_head(score, head, head)),
                             self.ds16, self.k, self.dq, C.CAUSAL_LEFT_MASKED),
            "dK": self._args(MatmulSpec.new(S, d, S).left_transposed().scaled(self.scale)
                             .batched(per_head(score, head, head)), self.ds16, self.q, self.dk, C.CAUSAL_LEFT_T_MASKED),
        }
        self.flops = product_flops(s)
        self.bytes = algorithmic_bytes(s)

    def _args(self, spec: MatmulSpec, left, right, out, causal: int) -> _ffi.GemmArgs:
        a = _ffi.GemmArgs()
        a.product = spec.product()
        a.count = spec.batch.count
        a.left_type = a.right_type = _ffi.TYPE_BF16
        a.output_type = _ffi.TYPE_F32
        a.precision = _ffi.PRECISION_BF16
        a.aux_type = _ffi.TYPE_F32
        a.left, a.left_len = left.data_ptr(), left.numel()
        a.right, a.right_len = right.data_ptr(), right.numel()
        a.output, a.output_len = out.data_ptr(), out.numel()
        a.causal = causal
        a.causal_offset = self.shape.query_offset
        return a

    def _gemm(self, h, name) -> None:
        check(self.lib.snb_gemm(h, ctypes.byref(self.args[name])))

    def forward(self, stream_handle: int) -> None:
        s = self.shape
        h = ctypes.c_void_p(stream_handle)
        self._gemm(h, "scores")
        check(self.lib.snb_causal_softmax_bf16(h, self.scores.data_ptr(), self.scores.numel(), s.count * s.time,
                                               s.time, s.time, self.scale, s.query_offset, self.p16.data_ptr()))
        self._gemm(h, "ctx")

    def backward(self, stream_handle: int) -> None:
        s = self.shape
        h = ctypes.c_void_p(stream_handle)
        self._gemm(h, "dP")
        self._gemm(h, "dV")
        check(self.lib.snb_causal_softmax_backward(h, self.scores.data_ptr(), self.d_scores.data_ptr(),
                                                   s.count * s.time, s.time, s.time, s.query_offset,
                                                   self.ds16.data_ptr()))
        self._gemm(h, "dQ")
        self._gemm(h, "dK")

    def launches(self) -> int:
        return 8


def fused_algorithmic_bytes(s: AttentionShape) -> float:
    """Bytes the fused forward + backward must move: Q, K, V, dO read (bf16), the f32 output and log-sum-exp written
    by the forward and read back by the backward, dQ, dK, dV written (f32)."""
    n, S, d = s.count, s.time, s.head_dim
    head = S * d
    fwd = 3 * head * 2 + head * 4 + S * 4
    bwd = 4 * head * 2 + head * 4 + S * 4 + 3 * head * 4
    return float(n) * (fwd + bwd)


class FusedAttention:
    """The same attention layer call through the fused entry points: snb_causal_attention_forward (output f32 and
    log-sum-exp) and snb_causal_attention_backward (dQ, dK, dV f32), on head-major tensors [batch*heads, time, 64].
    No [time, time] tensor exists; the backward recomputes the scores (one product more than the materialised six,
    not counted in `flops`)."""

    def __init__(self, shape: AttentionShape, device, seed: int = 0):
        import torch

        s = shape
        self.shape = s
        n, S, d = s.count, s.time, s.head_dim
        # Q, K, V and dO from the reference's generator (Random::new(seed), random.rs:27-70), drawn on the device.
        rng = DeviceRandom(Gpu(device.index if device.index is not None else 0), seed)

        def normal():
            return rng.normal_(torch.empty(n, S, d, device=device, dtype=torch.bfloat16))

        self.q, self.k, self.v, self.d_out = (normal() for _ in range(4))
        self.out = torch.empty(n, S, d, device=device, dtype=torch.float32)
        self.lse = torch.empty(n, S, device=device, dtype=torch.float32)
        self.dq, self.dk, self.dv = (torch.empty(n, S, d, device=device, dtype=torch.float32) for _ in range(3))
        self.scale = 1.0 / (d ** 0.5)
        self.gpu = Gpu(device.index if device.index is not None else 0)
        self.flops = product_flops(s)
        self.backward_flops = 5 * 2.0 * s.head_dim * causal_pairs(s) * s.count
        self.bytes = fused_algorithmic_bytes(s)

    def forward(self, stream_handle: int = 0) -> None:
        self.gpu.causal_attention_forward(self.q, self.k, self.v, self.out, self.scale, self.shape.query_offset,
                                          self.lse)

    def backward(self, stream_handle: int = 0) -> None:
        self.gpu.causal_attention_backward(self.q, self.k, self.v, self.out, self.d_out, self.lse, self.dq, self.dk,
                                           self.dv, self.scale, self.shape.query_offset)

    def launches(self) -> int:
        """Kernels of one forward + backward: the forward kernel, the row-statistics and backward kernels."""
        return 3


@dataclass(frozen=True)
class LayerShape:
    """Geometry of one attention layer call: `batch` sequences of `time` steps, `heads` heads of `head_dim`."""

    batch: int = 32
    time: int = 2048
    heads: int = 12
    head_dim: int = 64

    @property
    def width(self) -> int:
        return self.heads * self.head_dim

    @property
    def tokens(self) -> int:
        return self.batch * self.time


class CausalSelfAttentionLayer:
    """`CausalSelfAttention::forward` / `backward` (crates/staleynet-model/src/layers/attention.rs:188-267) on the C
    ABI, bf16 activations and weights W[in, out] (the reference's layout), f32 weight gradients.

    With fused_permutes (the default) the reference's head permutes run inside the products around attention:
      forward   qkv     = x Wqkv + b, written head-major (snb_gemm output_heads: the three split_heads,
                          attention.rs:201-204)
                o, lse  = causal attention of q, k, v (snb_causal_attention_forward: QK^T, causal_softmax, P V,
                          attention.rs:206-213)
                y       = o Wo + b, o read head-major (snb_gemm left_heads: merge_heads, attention.rs:214-216)
      backward  dWo    += o^T dy, o read head-major                      (Linear::backward, linear.rs:55-58)
                do      = dy Wo^T, written head-major (output_heads: split_heads of the context gradient,
                          attention.rs:233-237)
                dq, dk, dv = snb_causal_attention_backward                (attention.rs:239-260)
                dqkv    = the three merge_heads, f32 -> bf16 (snb_permute_heads, attention.rs:262-264)
                dWqkv  += x^T dqkv ;  dx = dqkv Wqkv^T                    (attention.rs:266, linear.rs:51-63)
    Without it, the products write and read packed tensors and snb_permute_heads moves the heads in between, as the
    reference does. Bias gradients (column sums of dy, not products) are not computed here."""

    def __init__(self, shape: LayerShape, device, seed: int = 0, fused_permutes: bool = True,
                 deterministic: bool = False):
        import torch

        s = shape
        self.shape = s
        self.fused = fused_permutes
        self.deterministic = deterministic
        self.gpu = Gpu(device.index if device.index is not None else 0)
        T, w, n, S, d = s.tokens, s.width, s.batch * s.heads, s.time, s.head_dim
        bf16, f32 = torch.bfloat16, torch.float32
        rng = DeviceRandom(self.gpu, seed)
        std = 1.0 / (w ** 0.5)
        self.w_qkv = rng.normal_(torch.empty(w, 3 * w, device=device, dtype=bf16), std)
        self.b_qkv = rng.normal_(torch.empty(3 * w, device=device, dtype=f32), 0.1)
        self.w_o = rng.normal_(torch.empty(w, w, device=device, dtype=bf16), std)
        self.b_o = rng.normal_(torch.empty(w, device=device, dtype=f32), 0.1)
        self.g_wqkv = torch.zeros(w, 3 * w, device=device, dtype=f32)
        self.g_wo = torch.zeros(w, w, device=device, dtype=f32)
        self.qkv_heads = torch.empty(3, n, S, d, device=device, dtype=bf16)   # q, k, v head-major
        self.o_heads = torch.empty(n, S, d, device=device, dtype=bf16)        # attention output (context)
        self.lse = torch.empty(n, S, device=device, dtype=f32)
        self.do_heads = torch.empty(n, S, d, device=device, dtype=bf16)
        self.dq, self.dk, self.dv = (torch.empty(n, S, d, device=device, dtype=f32) for _ in range(3))
        self.d_qkv = torch.empty(T, 3 * w, device=device, dtype=bf16)
        if not fused_permutes:
            self.qkv = torch.empty(T, 3 * w, device=device, dtype=bf16)
            self.o = torch.empty(T, w, device=device, dtype=bf16)
            self.d_o = torch.empty(T, w, device=device, dtype=bf16)
        self.scale = 1.0 / (d ** 0.5)

    def layout(self, width: int, column_offset: int) -> _ffi.HeadLayout:
        """`CausalSelfAttention::layout` (attention.rs:170-173): a projection's heads in a packed row of `width`."""
        s = self.shape
        return _ffi.HeadLayout.dense(s.batch, s.time, s.heads, s.head_dim, width, column_offset)

    def forward(self, x, y) -> None:
        """y [tokens, width] (bf16) = the layer's output for x [tokens, width] (bf16)."""
        s, g = self.shape, self.gpu
        T, w = s.tokens, s.width
        if self.fused:
            g.gemm(MatmulSpec.new(T, 3 * w, w), x, self.w_qkv, self.qkv_heads, bias=self.b_qkv,
                   output_heads=self.layout(3 * w, 0))
        else:
            g.gemm(MatmulSpec.new(T, 3 * w, w), x, self.w_qkv, self.qkv, bias=self.b_qkv)
            for p in range(3):
                g.split_heads(self.qkv, self.qkv_heads[p], self.layout(3 * w, p * w))
        q, k, v = self.qkv_heads
        g.causal_attention_forward(q, k, v, self.o_heads, self.scale, 0, self.lse)
        if self.fused:
            g.gemm(MatmulSpec.new(T, w, w), self.o_heads, self.w_o, y, bias=self.b_o, left_heads=self.layout(w, 0))
        else:
            g.merge_heads(self.o_heads, self.o, self.layout(w, 0))
            g.gemm(MatmulSpec.new(T, w, w), self.o, self.w_o, y, bias=self.b_o)

    def backward(self, x, dy, dx) -> None:
        """Accumulates g_wqkv and g_wo and writes dx [tokens, width] (bf16) for the output gradient dy (bf16)."""
        s, g = self.shape, self.gpu
        T, w = s.tokens, s.width
        det = self.deterministic
        if self.fused:
            g.gemm(MatmulSpec.new(w, w, T).left_transposed().accumulate(), self.o_heads, dy, self.g_wo,
                   left_heads=self.layout(w, 0), deterministic=det)
            g.gemm(MatmulSpec.new(T, w, w).right_transposed(), dy, self.w_o, self.do_heads,
                   output_heads=self.layout(w, 0))
        else:
            g.gemm(MatmulSpec.new(w, w, T).left_transposed().accumulate(), self.o, dy, self.g_wo, deterministic=det)
            g.gemm(MatmulSpec.new(T, w, w).right_transposed(), dy, self.w_o, self.d_o)
            g.split_heads(self.d_o, self.do_heads, self.layout(w, 0))
        q, k, v = self.qkv_heads
        g.causal_attention_backward(q, k, v, self.o_heads, self.do_heads, self.lse, self.dq, self.dk, self.dv,
                                    self.scale, 0)
        for p, grad in enumerate((self.dq, self.dk, self.dv)):
            g.merge_heads(grad, self.d_qkv, self.layout(3 * w, p * w))
        g.gemm(MatmulSpec.new(w, 3 * w, T).left_transposed().accumulate(), x, self.d_qkv, self.g_wqkv,
               deterministic=det)
        g.gemm(MatmulSpec.new(T, w, 3 * w).right_transposed(), self.d_qkv, self.w_qkv, dx)
