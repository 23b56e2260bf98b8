"""Host-side mirror of the reference's GEMM operator API (crates/staleynet-cuda/src/ops/matmul.rs, ops/mod.rs,
device.rs), bound to the sm_100a library through the C ABI.

Names, fields and error behaviour follow the reference so callers and tests read like the reference's own:
`Storage`, `BatchStrides`, `MatmulSpec` with its builders, `WriteMode`, `MatmulKernel` with `tolerance()`, and
`Gpu.matmul(spec, left, right, output)`. Tensors are torch CUDA tensors (torch is the device-memory plumbing here);
every product runs in libsnb_b200.so.
"""
from __future__ import annotations

import ctypes
import enum
from dataclasses import dataclass, replace

from . import _ffi


class WriteMode(enum.Enum):
    """Overwrite or accumulate into the output (ops/mod.rs:27-45)."""

    OVERWRITE = 0
    ACCUMULATE = 1

    def flag(self) -> int:
        return self.value


class Storage(enum.Enum):
    """How an operand is laid out relative to the logical matrix op(X) (ops/matmul.rs:14-33)."""

    ROW_MAJOR = 0
    TRANSPOSED = 1

    def operand(self, rows: int, cols: int, batch_stride: int) -> _ffi.Operand:
        if self is Storage.ROW_MAJOR:
            return _ffi.Operand(row_stride=cols, col_stride=1, batch_stride=batch_stride)
        return _ffi.Operand(row_stride=1, col_stride=rows, batch_stride=batch_stride)


@dataclass(frozen=True)
class BatchStrides:
    """Element offsets between consecutive matrices of a batch (ops/matmul.rs:35-54)."""

    count: int
    left: int
    right: int
    output: int


BatchStrides.SINGLE = BatchStrides(count=1, left=0, right=0, output=0)


@dataclass(frozen=True)
class MatmulSpec:
    """Full description of one (batched) GEMM (ops/matmul.rs:56-142)."""

    rows: int
    cols: int
    inner: int
    left: Storage = Storage.ROW_MAJOR
    right: Storage = Storage.ROW_MAJOR
    batch: BatchStrides = BatchStrides.SINGLE
    scale: float = 1.0
    write: WriteMode = WriteMode.OVERWRITE

    @staticmethod
    def new(rows: int, cols: int, inner: int) -> "MatmulSpec":
        return MatmulSpec(rows, cols, inner)

    def left_transposed(self) -> "MatmulSpec":
        return replace(self, left=Storage.TRANSPOSED)

    def right_transposed(self) -> "MatmulSpec":
        return replace(self, right=Storage.TRANSPOSED)

    def accumulate(self) -> "MatmulSpec":
        return replace(self, write=WriteMode.ACCUMULATE)

    def scaled(self, scale: float) -> "MatmulSpec":
        return replace(self, scale=scale)

    def batched(self, strides: BatchStrides) -> "MatmulSpec":
        return replace(self, batch=strides)

    def product(self) -> _ffi.Product:
        """The kernel-level description (`MatmulSpec::product`, ops/matmul.rs:124-136)."""
        return _ffi.Product(
            rows=self.rows,
            cols=self.cols,
            inner=self.inner,
            left=self.left.operand(self.rows, self.inner, self.batch.left),
            right=self.right.operand(self.inner, self.cols, self.batch.right),
            output_batch_stride=self.batch.output,
            scale=self.scale,
            accumulate=self.write.flag(),
        )

    def required_len(self, stride: int, per_matrix: int) -> int:
        """Elements an operand of `per_matrix` elements must hold (ops/matmul.rs:138-141)."""
        return (self.batch.count - 1) * stride + per_matrix


EMPTY_TOKEN = 0xFFFFFFFF   # a missing target (crates/staleynet-cuda/src/kernels/mod.rs:46)


@dataclass(frozen=True)
class CrossEntropyHead:
    """`CrossEntropyHead` (crates/staleynet-cuda/src/ops/loss.rs:14-30): which logit columns and which target of each
    row one classifier owns."""

    column_offset: int
    classes: int
    target_stride: int
    target_offset: int
    grad_scale: float


@dataclass(frozen=True)
class AdamWHyperparameters:
    """`AdamWHyperparameters` (crates/staleynet-cuda/src/ops/optimizer.rs:9-28)."""

    learning_rate: float
    beta1: float
    beta2: float
    epsilon: float
    weight_decay: float
    step: int


class MatmulKernel(enum.Enum):
    """Arithmetic of `Gpu.matmul` (device.rs:38-67). The reference's four f32 kernels become two precisions of
    one sm_100a implementation; BF16_TENSOR_CORE is new and needs bf16 operands."""

    NAIVE = "naive"
    TILED = "tiled"
    BLOCKED = "blocked"
    TENSOR_CORE = "tensor_core"
    BF16_TENSOR_CORE = "bf16_tensor_core"

    def precision(self) -> int:
        if self is MatmulKernel.TENSOR_CORE:
            return _ffi.PRECISION_TF32
        if self is MatmulKernel.BF16_TENSOR_CORE:
            return _ffi.PRECISION_BF16
        return _ffi.PRECISION_F32

    def tolerance(self) -> float:
        """Largest max|delta|/max|expected| against an exact f32 product (device.rs:57-66); bf16 keeps 8
        mantissa bits, so its bound is the 1e-2 stated for bf16 in the build's north star."""
        if self is MatmulKernel.TENSOR_CORE:
            return 2e-3
        if self is MatmulKernel.BF16_TENSOR_CORE:
            return 1e-2
        return 1e-5


class SnbError(RuntimeError):
    """A failed library call: `code` is the SNB_ERR_* status, the message is snb_last_error()."""

    def __init__(self, code: int, message: str):
        super().__init__(f"{message} (status {code})")
        self.code = code


class OperandTooSmall(SnbError, AssertionError):
    """The reference's `assert!` panics on undersized operands (ops/matmul.rs:147-149)."""


def check(code: int) -> None:
    if code == _ffi.OK:
        return
    msg = _ffi.last_error()
    if code in (_ffi.ERR_LEFT_TOO_SMALL, _ffi.ERR_RIGHT_TOO_SMALL, _ffi.ERR_OUTPUT_TOO_SMALL):
        raise OperandTooSmall(code, msg)
    raise SnbError(code, msg)


def _ptr(t) -> int:
    return int(t.data_ptr()) if t is not None else 0


def _require_cuda(*tensors) -> None:
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise SnbError(_ffi.ERR_INVALID_ARGUMENT, "tensors must live in CUDA device memory")


class Gpu:
    """One device and one stream, like the reference's `Gpu` (device.rs:129-208). `matmul_kernel` selects the
    arithmetic (the reference's `--matmul` switch)."""

    def __init__(self, device: int = 0, stream=None):
        import torch

        self.device = torch.device("cuda", device)
        self.stream = stream if stream is not None else torch.cuda.current_stream(self.device)
        self.matmul_kernel = MatmulKernel.BLOCKED
        self.lib = _ffi.load()

    def _stream_handle(self):
        return ctypes.c_void_p(self.stream.cuda_stream)

    def matmul(self, spec: MatmulSpec, left, right, output) -> None:
        """`Gpu::matmul` (ops/matmul.rs:146-171): output[b] = scale*op(left[b])*op(right[b]) (+ output[b])."""
        import torch

        _require_cuda(left, right, output)
        product = spec.product()
        if self.matmul_kernel is MatmulKernel.BF16_TENSOR_CORE:
            if left.dtype != torch.bfloat16 or right.dtype != torch.bfloat16 or output.dtype != torch.float32:
                raise SnbError(_ffi.ERR_INVALID_ARGUMENT, "bf16 matmul takes bf16 operands and an f32 output")
            code = self.lib.snb_matmul_bf16(self._stream_handle(), ctypes.byref(product), spec.batch.count,
                                            _ptr(left), left.numel(), _ptr(right), right.numel(), _ptr(output),
                                            output.numel())
        else:
            if left.dtype != torch.float32 or right.dtype != torch.float32 or output.dtype != torch.float32:
                raise SnbError(_ffi.ERR_INVALID_ARGUMENT, "f32 matmul takes f32 tensors")
            code = self.lib.snb_matmul(self._stream_handle(), ctypes.byref(product), spec.batch.count, _ptr(left),
                                       left.numel(), _ptr(right), right.numel(), _ptr(output), output.numel(),
                                       self.matmul_kernel.precision())
        check(code)

    def gemm(self, spec: MatmulSpec, left, right, output, *, bias=None, activation: int = _ffi.ACTIVATION_NONE,
             pre_activation=None, gelu_input=None, residual=None, causal: int = _ffi.CAUSAL_NONE,
             causal_offset: int = 0, row_scale=None, deterministic: bool = False, left_heads=None,
             output_heads=None) -> None:
        """`Gpu.matmul` with the caller's elementwise follow-up fused into the epilogue (snb_gemm). deterministic:
        split-K partial sums added in a fixed order (SNB_GEMM_DETERMINISTIC), bit-identical between runs.
        left_heads / output_heads (HeadLayout): the left operand is read from, or the output written to, the
        head-major form of the packed tensor the spec describes (the split/merge permutes fused into the product)."""
        args = self.gemm_args(spec, left, right, output, bias=bias, activation=activation,
                              pre_activation=pre_activation, gelu_input=gelu_input, residual=residual, causal=causal,
                              causal_offset=causal_offset, row_scale=row_scale, deterministic=deterministic,
                              left_heads=left_heads, output_heads=output_heads)
        check(self.lib.snb_gemm(self._stream_handle(), ctypes.byref(args)))

    def gemm_args(self, spec: MatmulSpec, left, right, output, *, bias=None, activation: int = _ffi.ACTIVATION_NONE,
                  pre_activation=None, gelu_input=None, residual=None, causal: int = _ffi.CAUSAL_NONE,
                  causal_offset: int = 0, row_scale=None, deterministic: bool = False, left_heads=None,
                  output_heads=None) -> _ffi.GemmArgs:
        """The snb_gemm_args of `gemm` (for entry points that take a GEMM as an argument)."""
        import torch

        _require_cuda(left, right, output, bias, pre_activation, gelu_input, residual)
        bf16 = left.dtype == torch.bfloat16
        args = _ffi.GemmArgs()
        args.product = spec.product()
        args.count = spec.batch.count
        args.left_type = args.right_type = _ffi.TYPE_BF16 if bf16 else _ffi.TYPE_F32
        if right.dtype != left.dtype:
            raise SnbError(_ffi.ERR_INVALID_ARGUMENT, "left and right must share a dtype")
        args.output_type = _ffi.TYPE_BF16 if output.dtype == torch.bfloat16 else _ffi.TYPE_F32
        args.precision = _ffi.PRECISION_BF16 if bf16 else self.matmul_kernel.precision()
        if not bf16 and args.precision == _ffi.PRECISION_BF16:
            args.precision = _ffi.PRECISION_TF32
        args.left, args.left_len = _ptr(left), left.numel()
        args.right, args.right_len = _ptr(right), right.numel()
        args.output, args.output_len = _ptr(output), output.numel()
        args.bias = _ptr(bias) if bias is not None else None
        args.activation = activation
        aux = pre_activation if pre_activation is not None else gelu_input
        args.aux_type = _ffi.TYPE_BF16 if (aux is not None and aux.dtype == torch.bfloat16) else _ffi.TYPE_F32
        args.pre_activation = _ptr(pre_activation) if pre_activation is not None else None
        args.gelu_input = _ptr(gelu_input) if gelu_input is not None else None
        args.residual = _ptr(residual) if residual is not None else None
        args.causal = causal
        args.causal_offset = causal_offset
        args.row_scale = _ptr(row_scale) if row_scale is not None else None
        args.flags = _ffi.GEMM_DETERMINISTIC if deterministic else 0
        # The layouts must outlive the call: keep them on the argument block.
        args._heads = (left_heads, output_heads)
        args.left_heads = ctypes.pointer(left_heads) if left_heads is not None else None
        args.output_heads = ctypes.pointer(output_heads) if output_heads is not None else None
        return args

    def cross_entropy(self, logits, targets, head: "CrossEntropyHead", losses, logits_grad) -> None:
        """`Gpu::cross_entropy` (ops/loss.rs:35-71): per-row losses and this head's gradient columns, f32."""
        import torch

        _require_cuda(logits, targets, losses, logits_grad)
        if logits_grad.shape != logits.shape:
            raise AssertionError("cross_entropy: gradient shape")
        rows, cols = logits.shape
        t = targets if targets.dtype == torch.int32 else targets.to(torch.int32)
        h = _ffi.CrossEntropyHead(head.column_offset, head.classes, head.target_stride, head.target_offset,
                                  head.grad_scale, 0)
        code = self.lib.snb_cross_entropy(self._stream_handle(), _ptr(logits), rows, cols, _ptr(t), t.numel(),
                                          ctypes.byref(h), _ptr(losses), losses.numel(), _ptr(logits_grad))
        if code == _ffi.ERR_INVALID_ARGUMENT:
            raise AssertionError(self.lib.snb_last_error().decode())
        check(code)

    def rms_norm_forward(self, input, gain, output, inv_rms, epsilon: float) -> None:
        """`Gpu::rms_norm_forward` (ops/normalization.rs): f32 [rows, cols] rows normalised by 1/rms, times gain."""
        _require_cuda(input, gain, output, inv_rms)
        if output.shape != input.shape:
            raise AssertionError("rms_norm_forward: output shape")
        rows, cols = input.shape
        code = self.lib.snb_rms_norm_forward(self._stream_handle(), _ptr(input), rows, cols, _ptr(gain), gain.numel(),
                                             _ptr(output), _ptr(inv_rms), inv_rms.numel(), epsilon)
        if code == _ffi.ERR_INVALID_ARGUMENT:
            raise AssertionError(self.lib.snb_last_error().decode())
        check(code)

    def rms_norm_backward(self, output_grad, input, gain, inv_rms, input_grad, gain_grad) -> None:
        """`Gpu::rms_norm_backward`: input_grad written, gain_grad added to."""
        _require_cuda(output_grad, input, gain, inv_rms, input_grad, gain_grad)
        if output_grad.shape != input.shape:
            raise AssertionError("rms_norm_backward: output_grad shape")
        if input_grad.shape != input.shape:
            raise AssertionError("rms_norm_backward: input_grad shape")
        rows, cols = input.shape
        code = self.lib.snb_rms_norm_backward(self._stream_handle(), _ptr(output_grad), _ptr(input), _ptr(gain),
                                              _ptr(inv_rms), _ptr(input_grad), _ptr(gain_grad), gain_grad.numel(),
                                              rows, cols)
        if code == _ffi.ERR_INVALID_ARGUMENT:
            raise AssertionError(self.lib.snb_last_error().decode())
        check(code)

    def rms_norm_stats(self, input, epsilon: float, inv_rms, gain=None, output=None) -> None:
        """snb_rms_norm_stats: 1/rms per row of input (f32 or bf16), and the normalised rows when `output` is
        given."""
        import torch

        _require_cuda(input, inv_rms, gain, output)
        rows, cols = input.shape
        t = lambda x: _ffi.TYPE_BF16 if x.dtype == torch.bfloat16 else _ffi.TYPE_F32  # noqa: E731
        check(self.lib.snb_rms_norm_stats(self._stream_handle(), _ptr(input), t(input), rows, cols, epsilon,
                                          _ptr(inv_rms), _ptr(gain) if gain is not None else None,
                                          _ptr(output) if output is not None else None,
                                          t(output) if output is not None else _ffi.TYPE_F32))

    def scale_rows(self, scale, input, output) -> None:
        """snb_scale_rows: output[k, :] = scale[k] * input[k, :]."""
        import torch

        _require_cuda(scale, input, output)
        rows, cols = input.shape
        t = lambda x: _ffi.TYPE_BF16 if x.dtype == torch.bfloat16 else _ffi.TYPE_F32  # noqa: E731
        check(self.lib.snb_scale_rows(self._stream_handle(), _ptr(scale), _ptr(input), t(input), _ptr(output),
                                      t(output), rows, cols))

    def adamw_step(self, parameter, gradient, first_moment, second_moment, hyper: "AdamWHyperparameters") -> None:
        """`Gpu::adamw_step` (ops/optimizer.rs:32-66)."""
        _require_cuda(parameter, gradient, first_moment, second_moment)
        if not (gradient.shape == parameter.shape == first_moment.shape == second_moment.shape):
            raise AssertionError("adamw_step: shape mismatch")
        h = _ffi.AdamWHyper(hyper.learning_rate, hyper.beta1, hyper.beta2, hyper.epsilon, hyper.weight_decay,
                            hyper.step)
        check(self.lib.snb_adamw_step(self._stream_handle(), _ptr(parameter), _ptr(gradient), _ptr(first_moment),
                                      _ptr(second_moment), parameter.numel(), ctypes.byref(h)))

    def random_normal(self, output, seed: int, first_draw: int = 0, std: float = 1.0) -> int:
        """snb_random_normal: `output` (f32 or bf16) = std * normal() of the reference's `Random::new(seed)` after
        `first_draw` draws (random.rs:27-70, two draws per value). Returns the draw count after the fill."""
        import torch

        _require_cuda(output)
        if output.dtype not in (torch.float32, torch.bfloat16):
            raise SnbError(_ffi.ERR_INVALID_ARGUMENT, "random_normal: output must be float32 or bfloat16")
        out_type = _ffi.TYPE_BF16 if output.dtype == torch.bfloat16 else _ffi.TYPE_F32
        check(self.lib.snb_random_normal(self._stream_handle(), _ptr(output), out_type, output.numel(),
                                         seed & 0xFFFFFFFFFFFFFFFF, first_draw, std))
        return first_draw + 2 * output.numel()

    def random_below(self, output, bound: int, seed: int, first_draw: int = 0) -> int:
        """snb_random_below: `output` (int32, read as uint32) = `Random::below(bound)` of `Random::new(seed)` after
        `first_draw` draws (random.rs:54-56). Returns the draw count after the fill."""
        import torch

        _require_cuda(output)
        if output.dtype != torch.int32:
            raise SnbError(_ffi.ERR_INVALID_ARGUMENT, "random_below: output must be int32")
        check(self.lib.snb_random_below(self._stream_handle(), _ptr(output), output.numel(),
                                        seed & 0xFFFFFFFFFFFFFFFF, first_draw, bound))
        return first_draw + output.numel()

    def sum_of_squares(self, values, result) -> None:
        """snb_sum_of_squares into a one-element float64 device tensor."""
        _require_cuda(values, result)
        check(self.lib.snb_sum_of_squares(self._stream_handle(), _ptr(values), values.numel(), _ptr(result)))

    def adamw_step_multi(self, tensors, hyper: "AdamWHyperparameters", max_gradient_norm: float,
                         gradient_square_sum) -> None:
        """snb_adamw_step_multi over [(parameter, gradient, first, second, weight_decay), ...]."""
        arr = (_ffi.AdamWTensor * max(1, len(tensors)))()
        for i, (p, g, m1, m2, wd) in enumerate(tensors):
            _require_cuda(p, g, m1, m2)
            arr[i] = _ffi.AdamWTensor(_ptr(p), _ptr(g), _ptr(m1), _ptr(m2), p.numel(), wd, 0)
        h = _ffi.AdamWHyper(hyper.learning_rate, hyper.beta1, hyper.beta2, hyper.epsilon, 0.0, hyper.step)
        check(self.lib.snb_adamw_step_multi(self._stream_handle(), arr, len(tensors), ctypes.byref(h),
                                            max_gradient_norm, _ptr(gradient_square_sum)))

    def head_cross_entropy(self, spec: MatmulSpec, x, w, logits, targets, codebooks: int, grad_scales, loss_sums,
                           logits_grad, *, bias=None) -> None:
        """The output layer's forward and per-codebook cross-entropy (snb_head_cross_entropy): logits = x w (+ bias)
        then, for every codebook c, loss_sums[c] = sum of its row losses and its gradient columns into logits_grad
        (which may be `logits` itself for an in-place gradient). targets: [rows, codebooks] int32/uint32 bits."""
        import torch

        _require_cuda(targets, grad_scales, loss_sums, logits_grad)
        args = self.gemm_args(spec, x, w, logits, bias=bias)
        t = targets if targets.dtype == torch.int32 else targets.to(torch.int32)
        grad_type = _ffi.TYPE_BF16 if logits_grad.dtype == torch.bfloat16 else _ffi.TYPE_F32
        check(self.lib.snb_head_cross_entropy(self._stream_handle(), ctypes.byref(args), _ptr(t), t.numel(),
                                              codebooks, spec.cols // codebooks, _ptr(grad_scales), _ptr(loss_sums),
                                              _ptr(logits_grad), grad_type))

    def codebook_cross_entropy(self, logits, targets, codebooks: int, grad_scales, loss_sums, logits_grad) -> None:
        """Every codebook's cross-entropy of logits [rows, codebooks * size] already computed
        (snb_codebook_cross_entropy): loss_sums[c] = sum of codebook c's row losses, its gradient into logits_grad
        (which may be `logits` itself). targets: [rows, codebooks] int32/uint32 bits."""
        import torch

        _require_cuda(logits, targets, grad_scales, loss_sums, logits_grad)
        t = targets if targets.dtype == torch.int32 else targets.to(torch.int32)
        rows = t.numel() // codebooks if logits.dim() == 1 else logits.shape[0]
        size = logits.numel() // rows // codebooks
        lt = _ffi.TYPE_BF16 if logits.dtype == torch.bfloat16 else _ffi.TYPE_F32
        gt = _ffi.TYPE_BF16 if logits_grad.dtype == torch.bfloat16 else _ffi.TYPE_F32
        check(self.lib.snb_codebook_cross_entropy(self._stream_handle(), _ptr(logits), lt, rows, codebooks, size,
                                                  _ptr(t), t.numel(), _ptr(grad_scales), _ptr(loss_sums),
                                                  _ptr(logits_grad), gt))

    def split_heads(self, packed, head_major, layout: "_ffi.HeadLayout") -> None:
        """`Gpu::split_heads` (crates/staleynet-cuda/src/ops/attention.rs:20-36): packed columns -> head-major; f32
        through snb_split_heads, other dtypes through snb_permute_heads."""
        self.permute_heads(_ffi.HEADS_SPLIT, packed, head_major, layout)

    def merge_heads(self, head_major, packed, layout: "_ffi.HeadLayout") -> None:
        """`Gpu::merge_heads` (ops/attention.rs:38-52): head-major -> packed columns, other columns untouched."""
        self.permute_heads(_ffi.HEADS_MERGE, head_major, packed, layout)

    def permute_heads(self, direction: int, src, dst, layout: "_ffi.HeadLayout") -> None:
        import torch

        _require_cuda(src, dst)
        h = self._stream_handle()
        if src.dtype == torch.float32 and dst.dtype == torch.float32:
            fn = self.lib.snb_split_heads if direction == _ffi.HEADS_SPLIT else self.lib.snb_merge_heads
            check(fn(h, _ptr(src), src.numel(), _ptr(dst), dst.numel(), ctypes.byref(layout)))
            return
        ty = {torch.float32: _ffi.TYPE_F32, torch.bfloat16: _ffi.TYPE_BF16}
        if src.dtype not in ty or dst.dtype not in ty:
            raise SnbError(_ffi.ERR_INVALID_ARGUMENT, "permute_heads: tensors must be float32 or bfloat16")
        check(self.lib.snb_permute_heads(h, direction, _ptr(src), ty[src.dtype], src.numel(), _ptr(dst),
                                         ty[dst.dtype], dst.numel(), ctypes.byref(layout)))

    def causal_softmax(self, scores, queries: int, scale: float, query_offset: int) -> None:
        """`Gpu::causal_softmax` (ops/attention.rs:57-81) on scores [rows, keys]."""
        _require_cuda(scores)
        rows, keys = scores.shape
        if rows % queries != 0:
            raise AssertionError("causal_softmax: rows must be a multiple of queries")
        check(self.lib.snb_causal_softmax(self._stream_handle(), _ptr(scores), scores.numel(), rows, queries, keys,
                                          scale, query_offset))

    def causal_softmax_bf16(self, scores, queries: int, scale: float, query_offset: int, probabilities_bf16) -> None:
        """causal_softmax that also writes the probabilities as bf16 (snb_causal_softmax_bf16)."""
        _require_cuda(scores, probabilities_bf16)
        rows, keys = scores.shape
        check(self.lib.snb_causal_softmax_bf16(self._stream_handle(), _ptr(scores), scores.numel(), rows, queries,
                                               keys, scale, query_offset, _ptr(probabilities_bf16)))

    def causal_softmax_backward(self, probabilities, grad, queries: int, query_offset: int, grad_bf16=None) -> None:
        """softmax_backward reading only the visible keys of causal probabilities (snb_causal_softmax_backward)."""
        _require_cuda(probabilities, grad, grad_bf16)
        rows, cols = probabilities.shape
        check(self.lib.snb_causal_softmax_backward(self._stream_handle(), _ptr(probabilities), _ptr(grad), rows,
                                                   queries, cols, query_offset,
                                                   _ptr(grad_bf16) if grad_bf16 is not None else None))

    def causal_attention_forward(self, q, k, v, out, scale: float, query_offset: int = 0, lse=None) -> None:
        """Fused causal attention forward (snb_causal_attention_forward): q [count, queries, 64], k/v
        [count, keys, 64] bf16; out f32 or bf16 [count, queries, 64]; lse f32 [count, queries] or None."""
        import torch

        _require_cuda(q, k, v, out, lse)
        count, queries, head_dim = q.shape
        keys = k.shape[1]
        out_type = _ffi.TYPE_BF16 if out.dtype == torch.bfloat16 else _ffi.TYPE_F32
        check(self.lib.snb_causal_attention_forward(self._stream_handle(), _ptr(q), _ptr(k), _ptr(v), count, queries,
                                                    keys, head_dim, scale, query_offset, _ptr(out), out_type,
                                                    _ptr(lse) if lse is not None else None))

    def causal_attention_backward(self, q, k, v, out, d_out, lse, dq, dk, dv, scale: float,
                                  query_offset: int = 0, no_alloc: bool = False) -> None:
        """Fused causal attention backward (snb_causal_attention_backward): q, d_out [count, queries, 64] and k, v
        [count, keys, 64] bf16; out (f32 or bf16) and lse as written by causal_attention_forward; dq, dk, dv f32,
        overwritten. no_alloc selects snb_causal_attention_backward_noalloc (static scratch, nothing allocated;
        overlapping calls on one device race on its scratch)."""
        import torch

        _require_cuda(q, k, v, out, d_out, lse, dq, dk, dv)
        count, queries, head_dim = q.shape
        keys = k.shape[1]
        out_type = _ffi.TYPE_BF16 if out.dtype == torch.bfloat16 else _ffi.TYPE_F32
        fn = self.lib.snb_causal_attention_backward_noalloc if no_alloc else self.lib.snb_causal_attention_backward
        check(fn(self._stream_handle(), _ptr(q), _ptr(k), _ptr(v), _ptr(out), out_type, _ptr(d_out), _ptr(lse), count,
                 queries, keys, head_dim, scale, query_offset, _ptr(dq), _ptr(dk), _ptr(dv)))

    def softmax_backward(self, probabilities, grad) -> None:
        """`Gpu::softmax_backward` (ops/attention.rs:83-100)."""
        _require_cuda(probabilities, grad)
        if tuple(probabilities.shape) != tuple(grad.shape):
            raise AssertionError("softmax_backward: shape mismatch")
        rows, cols = probabilities.shape
        check(self.lib.snb_softmax_backward(self._stream_handle(), _ptr(probabilities), _ptr(grad), rows, cols))

    def synchronize(self) -> None:
        self.stream.synchronize()

    def device_status(self) -> None:
        """Raises if a tensor-core kernel's bounded wait gave up since the last check."""
        check(self.lib.snb_device_status())


def last_path() -> int:
    return _ffi.last_path()


class DeviceRandom:
    """The reference's `Random::new(seed)` (crates/staleynet-model/src/random.rs:27-70) as a draw counter over the
    device fills: `normal_` and `below_` write what the same sequence of `Init::Normal(std)` / `below(bound)` calls
    would produce on the host, and advance the counter by the draws they consume."""

    def __init__(self, gpu: "Gpu", seed: int):
        self.gpu = gpu
        self.seed = seed
        self.draws = 0

    def normal_(self, output, std: float = 1.0):
        self.draws = self.gpu.random_normal(output, self.seed, self.draws, std)
        return output

    def below_(self, output, bound: int):
        self.draws = self.gpu.random_below(output, bound, self.seed, self.draws)
        return output
