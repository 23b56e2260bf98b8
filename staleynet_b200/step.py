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
and the output head (gpt.rs:72; training.rs:201-202, 247-248): logits = X·Wh + b, then every codebook's softmax
cross-entropy with its gradient dL written over the logits (training.rs:209-235, one launch, loss sums on the device),
then dWh += Xᵀ·dL, dX = dL·Whᵀ.

A step may cover several micro-batches (the reference's gradient accumulation: every dW product accumulates, and the
gradients are zeroed once per step), each a forward, loss and backward over its own input tokens and targets.
Inputs come from one seeded stream of the reference's generator: micro-batch g of the global batch takes the g-th
slice of it, so any rank can rebuild any micro-batch.

Attention scores, softmax and norms are not GEMMs of the linear stack and are not part of this workload (the
attention products are covered by the tests and by snb_causal_softmax); their activations are stood in for by
seeded tensors of the same shapes. Operands are bf16 with f32 accumulation (or f32 tensors on TF32 tensor cores or
the exact-f32 SIMT kernel); weight gradients accumulate in f32 through the tensor core's reduce-add epilogue;
activations and activation gradients are written in the operand type by the producing GEMM's epilogue.
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


# Seeds of the reference's generator (Random::new, random.rs:27-70) for the step's tensors. Weights and the
# attention stand-ins use WEIGHT_SEED on every rank (data-parallel replicas hold the same model); micro-batch g of the
# global batch draws its input activations and targets from slice g of the INPUT_SEED / TARGET_SEED streams.
WEIGHT_SEED = 1234
INPUT_SEED = 7
TARGET_SEED = 8


class TrainingStepGemms:
    """Device buffers and pre-built C-ABI argument blocks for every GEMM of one micro-batch's forward and backward,
    plus the loss between them; `run()` issues them for one micro-batch, `run_step()` for all of a step's.

    micro_batches: micro-batches this process runs per step, global indices first_micro_batch, +1, ... .
    grad_scale: the loss-gradient scale 1 / (valid targets x codebooks) of the whole step (all micro-batches of
    all ranks; training.rs:214-221); by default that of this process's micro-batches alone.
    deterministic: every product runs with SNB_GEMM_DETERMINISTIC (weight gradients bit-identical between runs).
    precision: SNB_PRECISION_BF16 (bf16 activations and weights, the default), SNB_PRECISION_TF32 or
    SNB_PRECISION_F32 (f32 tensors, as the reference holds them, device.rs:245-275, on TF32 tensor cores or on the
    exact-f32 SIMT kernel: the reference's MatmulKernel::TensorCore and ::Blocked, device.rs:38-67)."""

    def __init__(self, shape: ModelShape, device, seed: int = WEIGHT_SEED, micro_batches: int = 1,
                 first_micro_batch: int = 0, grad_scale: float | None = None, deterministic: bool = False,
                 precision: int = _ffi.PRECISION_BF16):
        import torch

        self.shape = shape
        self.device = device
        self.deterministic = deterministic
        self.precision = precision
        self.lib = _ffi.load()
        s = shape
        T, w, f, V = s.tokens, s.width, s.ffn, s.head_width
        f32 = torch.float32
        act = torch.bfloat16 if precision == _ffi.PRECISION_BF16 else f32   # element type of every tensor
        self.elem_type = _ffi.TYPE_BF16 if precision == _ffi.PRECISION_BF16 else _ffi.TYPE_F32
        self.gpu = Gpu(device.index if device.index is not None else 0)
        # Weights and stand-ins come from the reference's generator (Random::new(seed), random.rs:27-70), drawn on
        # the device in the order they are created here.
        rng = DeviceRandom(self.gpu, seed)

        def normal(n, std, dtype=act):
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
        self.acts = []
        for _ in range(s.blocks):
            self.acts.append({
                "ctx": normal(T * w, 1.0),      # attention context (stands in for the attention output)
                "qkv": torch.empty(T * 3 * w, device=device, dtype=act),
                "mid": torch.empty(T * w, device=device, dtype=act),
                "pre": torch.empty(T * f, device=device, dtype=act),
                "hid": torch.empty(T * f, device=device, dtype=act),
                "out": torch.empty(T * w, device=device, dtype=act),
            })
        self.logits = torch.empty(T * V, device=device, dtype=act)   # overwritten in place by the loss gradient
        # Gradient buffers (reused across blocks, as the reference's shared gradient workspace).
        self.g_x = torch.empty(T * w, device=device, dtype=act)
        self.g_mid = torch.empty(T * w, device=device, dtype=act)
        self.g_pre = torch.empty(T * f, device=device, dtype=act)
        self.g_ctx = torch.empty(T * w, device=device, dtype=act)
        self.g_qkv = normal(T * 3 * w, 1.0)  # attention's gradient w.r.t. the fused projection (stand-in)
        self.g_in = torch.empty(T * w, device=device, dtype=act)

        # The step's micro-batches: input activations and targets, resident on the device.
        self.micro_batches = micro_batches
        self.first_micro_batch = first_micro_batch
        self.inputs = torch.empty(micro_batches, T * w, device=device, dtype=act)
        self.targets = torch.empty(micro_batches, T * s.codebooks, device=device, dtype=torch.int32)
        for m in range(micro_batches):
            self.load_micro_batch(first_micro_batch + m, self.inputs[m], self.targets[m])
        self.x_in = self.inputs[0]
        if grad_scale is None:
            grad_scale = 1.0 / (T * micro_batches * s.codebooks)
        self.grad_scale = grad_scale
        self.grad_scales = torch.full((s.codebooks,), grad_scale, device=device, dtype=f32)
        self.loss_sums = torch.zeros(micro_batches, s.codebooks, device=device, dtype=f32)
        self.flops = step_flops(s)
        self._build_plan()

    def load_micro_batch(self, global_index: int, x, targets) -> None:
        """Fills x ([tokens * width], the step's element type) and targets ([tokens * codebooks] int32) with micro-batch `global_index`
        of the global batch: slice global_index of the input stream (N(0,1) activations) and of the target stream
        (`below(codebook_size)`, as the reference's bench draws targets, bench.rs:152-154)."""
        s = self.shape
        n_x = s.tokens * s.width
        n_t = s.tokens * s.codebooks
        self.gpu.random_normal(x, INPUT_SEED, first_draw=2 * n_x * global_index, std=1.0)
        self.gpu.random_below(targets, s.codebook_size, TARGET_SEED, first_draw=n_t * global_index)

    # ------------------------------------------------------------------------------------------------ plan
    def _args(self, spec: MatmulSpec, left, right, output, *, bias=None, activation=_ffi.ACTIVATION_NONE,
              pre=None, gelu_input=None, residual=None) -> _ffi.GemmArgs:
        import torch

        a = _ffi.GemmArgs()
        a.product = spec.product()
        a.count = spec.batch.count
        a.left_type = a.right_type = self.elem_type
        a.output_type = _ffi.TYPE_BF16 if output.dtype == torch.bfloat16 else _ffi.TYPE_F32
        a.precision = self.precision
        a.left, a.left_len = left.data_ptr(), left.numel()
        a.right, a.right_len = right.data_ptr(), right.numel()
        a.output, a.output_len = output.data_ptr(), output.numel()
        a.bias = bias.data_ptr() if bias is not None else None
        a.activation = activation
        a.aux_type = self.elem_type
        a.pre_activation = pre.data_ptr() if pre is not None else None
        a.gelu_input = gelu_input.data_ptr() if gelu_input is not None else None
        a.residual = residual.data_ptr() if residual is not None else None
        a.flags = _ffi.GEMM_DETERMINISTIC if self.deterministic else 0
        return a

    def use_input(self, x) -> None:
        """Points the step's first-block products at input activations `x` (same shape and type as x_in), so a
        caller can upload the next micro-batch's input into another buffer while this one runs."""
        assert x.numel() == self.x_in.numel() and x.dtype == self.x_in.dtype
        for a in self._input_args:
            a.left = x.data_ptr()
        for a in self._residual_args:
            a.residual = x.data_ptr()

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
        # Backward: the loss gradient dL has overwritten the logits (snb_codebook_cross_entropy between the passes).
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
        # Block 0's output product reads the input as its residual: repointed with the others.
        self._residual_args = [fwd[1][2]]
        self.forward_plan = fwd
        self.backward_plan = bwd
        self.plan = fwd + bwd
        self.plan_flops = sum(fl for _, fl, _ in self.plan)

    # ------------------------------------------------------------------------------------------------ run
    def launches_per_step(self) -> int:
        """GEMM launches of one micro-batch (the loss kernel is not counted)."""
        return len(self.plan)

    def use_micro_batch(self, m: int, x=None) -> None:
        """Points the products at local micro-batch m's input (or at `x`, a buffer holding it)."""
        self.use_input(self.inputs[m] if x is None else x)

    def run(self, stream_handle: int, on_block_done=None, events=None, micro_batch: int = 0, x=None) -> None:
        """Issues the forward, loss and backward of local micro-batch `micro_batch` on `stream_handle`.
        `on_block_done(b)` is called after the backward GEMMs of block b have been issued (the data-parallel step
        starts that block's all-reduce there). With `events` (a list of (start, end) CUDA event pairs, one per GEMM)
        each GEMM launch is bracketed for kernel timing."""
        self.use_micro_batch(micro_batch, x)
        h = ctypes.c_void_p(stream_handle)
        gemm = self.lib.snb_gemm
        ends = dict((n, b) for b, n in self.block_bwd_end) if on_block_done else {}
        nfwd = len(self.forward_plan)
        s = self.shape
        for i, (_, _, args) in enumerate(self.plan):
            if events is not None:
                events[i][0].record()
            code = gemm(h, ctypes.byref(args))
            if code != _ffi.OK:
                check(code)
            if events is not None:
                events[i][1].record()
            if i == nfwd - 1:
                # Every codebook's loss and its gradient, written over the logits (training.rs:209-235).
                code = self.lib.snb_codebook_cross_entropy(
                    h, self.logits.data_ptr(), self.elem_type, s.tokens, s.codebooks, s.codebook_size,
                    self.targets[micro_batch].data_ptr(), self.targets[micro_batch].numel(),
                    self.grad_scales.data_ptr(), self.loss_sums[micro_batch].data_ptr(), self.logits.data_ptr(),
                    self.elem_type)
                if code != _ffi.OK:
                    check(code)
            if on_block_done is not None and (i + 1 - nfwd) in ends:
                on_block_done(ends[i + 1 - nfwd])

    def run_step(self, stream_handle: int, on_block_done=None, events=None, inputs=None) -> None:
        """One optimizer step's worth of work: gradients zeroed, then every local micro-batch in turn, each
        accumulating into the weight gradients; `on_block_done` (the all-reduce hook) fires during the last one's
        backward only. `events`: one list of event pairs per micro-batch, or None. `inputs`: a callable m -> buffer
        holding micro-batch m's input (the end-to-end run's upload buffers), or None for the resident inputs."""
        self.zero_grads()
        last = self.micro_batches - 1
        for m in range(self.micro_batches):
            self.run(stream_handle, on_block_done=on_block_done if m == last else None,
                     events=events[m] if events is not None else None, micro_batch=m,
                     x=inputs(m) if inputs is not None else None)

    def capture(self, micro_batch: int = 0, x=None):
        """Captures `run()` of local micro-batch `micro_batch` (forward, loss, backward; no collective hook) into a
        CUDA graph and returns it (torch.cuda.CUDAGraph; `replay()` reissues every launch with one call). Every library
        call on the path is capturable: kernel launches, split-K zeroing (memset nodes) and the deterministic mode's
        stream-ordered workspace; per-device set-up happens on the first, uncaptured, run, so run() must have been
        called once before. The graph holds the operand pointers of the capture: one graph per input buffer."""
        import torch

        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            self.run(torch.cuda.current_stream().cuda_stream, micro_batch=micro_batch, x=x)
        return graph

    def zero_grads(self) -> None:
        self.grads.zero_()
