"""The GEMMs of one training step of StaleyNET's decoder, issued through the C ABI: the benchmark workload and the
data-parallel step.

Per block (crates/staleynet-model/src/layers/block.rs:160-216) the step runs, in the reference's order:
  forward   qkv      Y[T,3w]  = X·Wqkv + b                       (linear.rs:43-48)
            output   Y[T,w]   = C·Wo + b + X          (residual add, block.rs:182)
            expand   H[T,4w]  = GELU(X·W1 + b), pre kept          (feed_forward.rs:55-59)
            project  Y[T,w]   = H·W2 + b + X          (residual add, block.rs:188)
  backward  project  dW2 += Hᵀ·dY ;  dPre = (dY·W2ᵀ) ⊙ gelu'(pre)  (linear.rs:51-63, feed_forward.rs:68-75)
            expand   dW1 += Xᵀ·dPre ; dX = dPre·W1ᵀ
            output   dWo += Cᵀ·dY ;   dC = dY·Woᵀ
            qkv      dWqkv += Xᵀ·dQKV ; dX = dQKV·Wqkvᵀ
and the output head (gpt.rs:72; training.rs:201-202, 247-248): logits = X·Wh + b, dWh += Xᵀ·dL, dX = dL·Whᵀ.

Attention scores, softmax and norms are not GEMMs of the linear stack and are not part of this workload (the
attention products are covered by the tests and by snb_causal_softmax); their activations are stood in for by
seeded tensors of the same shapes. Operands are bf16 with f32 accumulation; weight gradients accumulate in f32
through the tensor core's reduce-add epilogue; activations and activation gradients are written in bf16 by the
producing GEMM's epilogue.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

from . import _ffi
from .data_parallel import GradientBuckets
from .matmul import DeviceRandom, Gpu, MatmulSpec, check


@dataclass(frozen=True)
class ModelShape:
    """Decoder geometry (12 blocks, width 768, FFN 3072, 16 codebooks x 1024)."""

    blocks: int = 12
    width: int = 768
    ffn: int = 3072
    codebooks: int = 16
    codebook_size: int = 1024
    tokens: int = 32 * 2048

    @property
    def head_width(self) -> int:
        return self.codebooks * self.codebook_size


def linear_shapes(s: ModelShape):
    """(name, inputs, outputs) of the linear layers of one block."""
    return [("qkv", s.width, 3 * s.width), ("output", s.width, s.width), ("expand", s.width, s.ffn),
            ("project", s.ffn, s.width)]


def step_flops(s: ModelShape) -> float:
    """2*M*N*K summed over fwd, dX and dW of every linear and the head (the reference's GFLOP/s convention,
    crates/staleynet-cli/src/commands/bench.rs:139)."""
    per_block = sum(2.0 * s.tokens * i * o for _, i, o in linear_shapes(s))
    head = 2.0 * s.tokens * s.width * s.head_width
    return 3.0 * (s.blocks * per_block + head)


class TrainingStepGemms:
    """Device buffers and pre-built C-ABI argument blocks for every GEMM of one step; `run()` issues them."""

    def __init__(self, shape: ModelShape, device, seed: int = 0):
        import torch

        self.shape = shape
        self.device = device
        self.lib = _ffi.load()
        s = shape
        T, w, f, V = s.tokens, s.width, s.ffn, s.head_width
        bf16, f32 = torch.bfloat16, torch.float32
        # Inputs and weights come from the reference's generator (Random::new(seed), random.rs:27-70), drawn on the
        # device in the order they are created here.
        rng = DeviceRandom(Gpu(device.index if device.index is not None else 0), seed)

        def normal(n, std, dtype=bf16):
            return rng.normal_(torch.empty(n, device=device, dtype=dtype), std)

        wstd = 1.0 / (w ** 0.5)
        self.weights = []
        self.weight_grads = []
        self.biases = []
        for _ in range(s.blocks):
            ws = {name: normal(i * o, wstd) for name, i, o in linear_shapes(s)}
            self.weights.append(ws)
            self.biases.append({name: torch.zeros(o, device=device, dtype=f32) for name, _, o in linear_shapes(s)})
        # Weight gradients of one block are views of one flat f32 buffer, so the data-parallel step all-reduces a
        # block with one collective.
        sizes = [i * o for _, i, o in linear_shapes(s)]
        self.grads = GradientBuckets([sizes] * s.blocks, w * V, device, f32)
        self.block_grad_flat = self.grads.flat
        for b in range(s.blocks):
            self.weight_grads.append({name: view for (name, _, _), view in zip(linear_shapes(s), self.grads.views[b])})
        self.head_w = normal(w * V, wstd)
        self.head_b = torch.zeros(V, device=device, dtype=f32)
        self.head_grad = self.grads.head

        # Activations kept per block, as a training step keeps them for the backward pass.
        self.x_in = normal(T * w, 1.0)  # the step's input activations (uploaded per step in the end-to-end run)
        self.acts = []
        for _ in range(s.blocks):
            self.acts.append({
                "ctx": normal(T * w, 1.0),      # attention context (stands in for the attention output)
                "qkv": torch.empty(T * 3 * w, device=device, dtype=bf16),
                "mid": torch.empty(T * w, device=device, dtype=bf16),
                "pre": torch.empty(T * f, device=device, dtype=bf16),
                "hid": torch.empty(T * f, device=device, dtype=bf16),
                "out": torch.empty(T * w, device=device, dtype=bf16),
            })
        self.logits = torch.empty(T * V, device=device, dtype=bf16)
        # Gradient buffers (reused across blocks, as the reference's shared gradient workspace).
        self.g_x = torch.empty(T * w, device=device, dtype=bf16)
        self.g_mid = torch.empty(T * w, device=device, dtype=bf16)
        self.g_pre = torch.empty(T * f, device=device, dtype=bf16)
        self.g_ctx = torch.empty(T * w, device=device, dtype=bf16)
        self.g_qkv = normal(T * 3 * w, 1.0)  # attention's gradient w.r.t. the fused projection (stand-in)
        self.g_in = torch.empty(T * w, device=device, dtype=bf16)
        self.flops = step_flops(s)
        self._build_plan()

    # ------------------------------------------------------------------------------------------------ plan
    def _args(self, spec: MatmulSpec, left, right, output, *, bias=None, activation=_ffi.ACTIVATION_NONE,
              pre=None, gelu_input=None, residual=None) -> _ffi.GemmArgs:
        import torch

        a = _ffi.GemmArgs()
        a.product = spec.product()
        a.count = spec.batch.count
        a.left_type = a.right_type = _ffi.TYPE_BF16
        a.output_type = _ffi.TYPE_BF16 if output.dtype == torch.bfloat16 else _ffi.TYPE_F32
        a.precision = _ffi.PRECISION_BF16
        a.left, a.left_len = left.data_ptr(), left.numel()
        a.right, a.right_len = right.data_ptr(), right.numel()
        a.output, a.output_len = output.data_ptr(), output.numel()
        a.bias = bias.data_ptr() if bias is not None else None
        a.activation = activation
        a.aux_type = _ffi.TYPE_BF16
        a.pre_activation = pre.data_ptr() if pre is not None else None
        a.gelu_input = gelu_input.data_ptr() if gelu_input is not None else None
        a.residual = residual.data_ptr() if residual is not None else None
        return a

    def use_input(self, x) -> None:
        """Points the step's first-block products at input activations `x` (same shape and type as x_in), so a
        caller can upload the next step's input into a second buffer while this step runs."""
        assert x.numel() == self.x_in.numel() and x.dtype == self.x_in.dtype
        for a in self._input_args:
            a.left = x.data_ptr()

    def _build_plan(self) -> None:
        s = self.shape
        T, w, f, V = s.tokens, s.width, s.ffn, s.head_width
        fwd, bwd = [], []
        x = self.x_in
        self._input_args = []   # the argument blocks that read the step's input activations
        for b in range(s.blocks):
            W, B, A = self.weights[b], self.biases[b], self.acts[b]
            fwd.append(("qkv.fwd", 2.0 * T * w * 3 * w,
                        self._args(MatmulSpec.new(T, 3 * w, w), x, W["qkv"], A["qkv"], bias=B["qkv"])))
            if b == 0:
                self._input_args.append(fwd[-1][2])
            fwd.append(("output.fwd", 2.0 * T * w * w,
                        self._args(MatmulSpec.new(T, w, w), A["ctx"], W["output"], A["mid"], bias=B["output"],
                                   residual=x)))
            fwd.append(("expand.fwd", 2.0 * T * w * f,
                        self._args(MatmulSpec.new(T, f, w), A["mid"], W["expand"], A["hid"], bias=B["expand"],
                                   activation=_ffi.ACTIVATION_GELU, pre=A["pre"])))
            fwd.append(("project.fwd", 2.0 * T * f * w,
                        self._args(MatmulSpec.new(T, w, f), A["hid"], W["project"], A["out"], bias=B["project"],
                                   residual=A["mid"])))
            x = A["out"]
        fwd.append(("head.fwd", 2.0 * T * w * V,
                    self._args(MatmulSpec.new(T, V, w), x, self.head_w, self.logits, bias=self.head_b)))
        self.final_x = x
        # Backward: the head's upstream gradient is the logits tensor itself (a synthetic loss whose gradient
        # has the logits' shape and magnitude).
        bwd.append(("head.dW", 2.0 * T * w * V,
                    self._args(MatmulSpec.new(w, V, T).left_transposed().accumulate(), x, self.logits,
                               self.head_grad)))
        bwd.append(("head.dX", 2.0 * T * V * w,
                    self._args(MatmulSpec.new(T, w, V).right_transposed(), self.logits, self.head_w, self.g_x)))
        self.block_bwd_end = []
        for b in reversed(range(s.blocks)):
            W, G, A = self.weights[b], self.weight_grads[b], self.acts[b]
            x_b = self.x_in if b == 0 else self.acts[b - 1]["out"]
            bwd.append(("project.dW", 2.0 * T * f * w,
                        self._args(MatmulSpec.new(f, w, T).left_transposed().accumulate(), A["hid"], self.g_x,
                                   G["project"])))
            bwd.append(("project.dX", 2.0 * T * w * f,
                        self._args(MatmulSpec.new(T, f, w).right_transposed(), self.g_x, W["project"], self.g_pre,
                                   activation=_ffi.ACTIVATION_GELU_GRAD, gelu_input=A["pre"])))
            bwd.append(("expand.dW", 2.0 * T * w * f,
                        self._args(MatmulSpec.new(w, f, T).left_transposed().accumulate(), A["mid"], self.g_pre,
                                   G["expand"])))
            bwd.append(("expand.dX", 2.0 * T * f * w,
                        self._args(MatmulSpec.new(T, w, f).right_transposed(), self.g_pre, W["expand"],
                                   self.g_mid, residual=self.g_x)))
            bwd.append(("output.dW", 2.0 * T * w * w,
                        self._args(MatmulSpec.new(w, w, T).left_transposed().accumulate(), A["ctx"], self.g_mid,
                                   G["output"])))
            bwd.append(("output.dX", 2.0 * T * w * w,
                        self._args(MatmulSpec.new(T, w, w).right_transposed(), self.g_mid, W["output"],
                                   self.g_ctx)))
            bwd.append(("qkv.dW", 2.0 * T * w * 3 * w,
                        self._args(MatmulSpec.new(w, 3 * w, T).left_transposed().accumulate(), x_b, self.g_qkv,
                                   G["qkv"])))
            if b == 0:
                self._input_args.append(bwd[-1][2])
            bwd.append(("qkv.dX", 2.0 * T * 3 * w * w,
                        self._args(MatmulSpec.new(T, w, 3 * w).right_transposed(), self.g_qkv, W["qkv"],
                                   self.g_in, residual=self.g_mid)))
            self.block_bwd_end.append((b, len(bwd)))
        self.forward_plan = fwd
        self.backward_plan = bwd
        self.plan = fwd + bwd
        self.plan_flops = sum(fl for _, fl, _ in self.plan)

    # ------------------------------------------------------------------------------------------------ run
    def launches_per_step(self) -> int:
        return len(self.plan)

    def run(self, stream_handle: int, on_block_done=None, events=None) -> None:
        """Issues every GEMM of the step on `stream_handle`. `on_block_done(b)` is called after the backward GEMMs
        of block b have been issued (the data-parallel step starts that block's all-reduce there). With `events`
        (a list of (start, end) CUDA event pairs, one per GEMM) each launch is bracketed for kernel timing."""
        h = ctypes.c_void_p(stream_handle)
        gemm = self.lib.snb_gemm
        ends = dict((n, b) for b, n in self.block_bwd_end) if on_block_done else {}
        nfwd = len(self.forward_plan)
        for i, (_, _, args) in enumerate(self.plan):
            if events is not None:
                events[i][0].record()
            code = gemm(h, ctypes.byref(args))
            if code != _ffi.OK:
                check(code)
            if events is not None:
                events[i][1].record()
            if on_block_done is not None and (i + 1 - nfwd) in ends:
                on_block_done(ends[i + 1 - nfwd])

    def zero_grads(self) -> None:
        self.grads.zero_()
