"""ctypes binding of the C ABI in include/snb_matmul.h (libsnb_b200.so).

The structures mirror the header field for field; `Product` is byte-identical to the reference's `repr(C)`
`Product` (crates/staleynet-cuda/src/kernels/matmul.rs:128-157). Loading fails loudly when the library has not
been built: there is no fallback implementation.
"""
from __future__ import annotations

import ctypes
import threading
from ctypes import POINTER, c_char_p, c_float, c_int, c_int32, c_uint16, c_uint32, c_uint64, c_void_p
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libsnb_b200.so"

PRECISION_F32 = 0
PRECISION_TF32 = 1
PRECISION_BF16 = 2

TYPE_F32 = 0
TYPE_BF16 = 1

ACTIVATION_NONE = 0
ACTIVATION_GELU = 1
ACTIVATION_GELU_GRAD = 2

CAUSAL_NONE = 0
CAUSAL_SKIP_MASKED_OUTPUT = 1
CAUSAL_LEFT_MASKED = 2
CAUSAL_LEFT_T_MASKED = 3

GEMM_DETERMINISTIC = 1   # snb_gemm_args.flags: split-K partials summed in a fixed order

HEADS_SPLIT = 0          # snb_permute_heads directions
HEADS_MERGE = 1

OK = 0
ERR_LEFT_TOO_SMALL = 1
ERR_RIGHT_TOO_SMALL = 2
ERR_OUTPUT_TOO_SMALL = 3
ERR_INVALID_ARGUMENT = 4
ERR_UNSUPPORTED = 5
ERR_CUDA = 6
ERR_DEVICE_TIMEOUT = 7

PATH_NONE = 0
PATH_TENSOR_CORE = 1
PATH_SIMT = 2
PATH_EMPTY = 3
PATH_TENSOR_CORE_PAIR = 4
TENSOR_CORE_PATHS = (PATH_TENSOR_CORE, PATH_TENSOR_CORE_PAIR)

EXPORTED_SYMBOLS = (
    "snb_matmul",
    "snb_matmul_bf16",
    "snb_gemm",
    "snb_set_deterministic",
    "snb_set_sm_budget",
    "snb_causal_softmax",
    "snb_softmax_backward",
    "snb_causal_softmax_bf16",
    "snb_causal_softmax_backward",
    "snb_last_error",
    "snb_last_path",
    "snb_device_status",
    "snb_causal_attention_forward",
    "snb_causal_attention_backward",
    "snb_causal_attention_backward_noalloc",
    "snb_cross_entropy",
    "snb_head_cross_entropy",
    "snb_codebook_cross_entropy",
    "snb_split_heads",
    "snb_merge_heads",
    "snb_permute_heads",
    "snb_rms_norm_forward",
    "snb_rms_norm_backward",
    "snb_rms_norm_stats",
    "snb_scale_rows",
    "snb_adamw_step",
    "snb_sum_of_squares",
    "snb_adamw_step_multi",
    "snb_random_normal",
    "snb_random_below",
    "snb_selftest_bounded_wait",
    "snb_abi_version",
)


class Operand(ctypes.Structure):
    _fields_ = [("row_stride", c_uint64), ("col_stride", c_uint64), ("batch_stride", c_uint64)]


class Product(ctypes.Structure):
    _fields_ = [
        ("rows", c_uint64),
        ("cols", c_uint64),
        ("inner", c_uint64),
        ("left", Operand),
        ("right", Operand),
        ("output_batch_stride", c_uint64),
        ("scale", c_float),
        ("accumulate", c_uint32),
    ]


class CrossEntropyHead(ctypes.Structure):
    """snb_cross_entropy_head: the reference's CrossEntropyHead (ops/loss.rs:14-30)."""
    _fields_ = [("column_offset", c_uint64), ("classes", c_uint64), ("target_stride", c_uint64),
                ("target_offset", c_uint64), ("grad_scale", c_float), ("reserved", c_uint32)]


class AdamWHyper(ctypes.Structure):
    """snb_adamw_hyper: the reference's AdamWHyperparameters (ops/optimizer.rs:9-28)."""
    _fields_ = [("learning_rate", c_float), ("beta1", c_float), ("beta2", c_float), ("epsilon", c_float),
                ("weight_decay", c_float), ("step", c_uint32)]


class AdamWTensor(ctypes.Structure):
    """snb_adamw_tensor."""
    _fields_ = [("parameter", c_void_p), ("gradient", c_void_p), ("first_moment", c_void_p),
                ("second_moment", c_void_p), ("count", c_uint64), ("weight_decay", c_float), ("reserved", c_uint32)]


class HeadLayout(ctypes.Structure):
    """snb_head_layout: the reference's `HeadLayout` (crates/staleynet-cuda/src/kernels/attention.rs:19-41), 8 x u64."""

    _fields_ = [(name, c_uint64) for name in ("batch", "time", "heads", "head_dim", "width", "column_offset",
                                               "time_capacity", "time_offset")]

    @staticmethod
    def dense(batch, time, heads, head_dim, width, column_offset) -> "HeadLayout":
        """`HeadLayout::dense` (kernels/attention.rs:62-64): capacity = time, offset 0."""
        return HeadLayout(batch, time, heads, head_dim, width, column_offset, time, 0)

    def in_cache(self, capacity, offset) -> "HeadLayout":
        """`HeadLayout::in_cache` (kernels/attention.rs:67-69): the same heads in a cache of `capacity` steps."""
        return HeadLayout(self.batch, self.time, self.heads, self.head_dim, self.width, self.column_offset, capacity,
                          offset)


class GemmArgs(ctypes.Structure):
    _fields_ = [
        ("product", Product),
        ("count", c_uint64),
        ("left_type", c_int32),
        ("right_type", c_int32),
        ("output_type", c_int32),
        ("precision", c_int32),
        ("left", c_void_p),
        ("left_len", c_uint64),
        ("right", c_void_p),
        ("right_len", c_uint64),
        ("output", c_void_p),
        ("output_len", c_uint64),
        ("bias", c_void_p),
        ("activation", c_int32),
        ("aux_type", c_int32),
        ("pre_activation", c_void_p),
        ("gelu_input", c_void_p),
        ("residual", c_void_p),
        ("causal", c_int32),
        ("flags", c_int32),
        ("causal_offset", ctypes.c_int64),
        ("row_scale", c_void_p),
        ("left_heads", POINTER(HeadLayout)),
        ("output_heads", POINTER(HeadLayout)),
    ]


assert ctypes.sizeof(Operand) == 24
assert ctypes.sizeof(Product) == 88
assert ctypes.sizeof(HeadLayout) == 64

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


def load() -> ctypes.CDLL:
    """Loads libsnb_b200.so and declares every entry point's signature."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"{LIB_PATH} is missing: build the sm_100a library with `python -m staleynet_b200.build`")
        lib = ctypes.CDLL(str(LIB_PATH))
        lib.snb_matmul.argtypes = [c_void_p, POINTER(Product), c_uint64, c_void_p, c_uint64, c_void_p, c_uint64,
                                   c_void_p, c_uint64, c_int32]
        lib.snb_matmul.restype = c_int
        lib.snb_matmul_bf16.argtypes = [c_void_p, POINTER(Product), c_uint64, c_void_p, c_uint64, c_void_p,
                                        c_uint64, c_void_p, c_uint64]
        lib.snb_matmul_bf16.restype = c_int
        lib.snb_gemm.argtypes = [c_void_p, POINTER(GemmArgs)]
        lib.snb_gemm.restype = c_int
        lib.snb_set_deterministic.argtypes = [c_int32]
        lib.snb_set_deterministic.restype = c_int
        lib.snb_set_sm_budget.argtypes = [c_int32]
        lib.snb_set_sm_budget.restype = c_int
        lib.snb_causal_softmax.argtypes = [c_void_p, c_void_p, c_uint64, c_uint64, c_uint64, c_uint64, c_float,
                                           c_uint64]
        lib.snb_causal_softmax.restype = c_int
        lib.snb_softmax_backward.argtypes = [c_void_p, c_void_p, c_void_p, c_uint64, c_uint64]
        lib.snb_softmax_backward.restype = c_int
        lib.snb_causal_softmax_bf16.argtypes = [c_void_p, c_void_p, c_uint64, c_uint64, c_uint64, c_uint64,
                                                c_float, c_uint64, c_void_p]
        lib.snb_causal_softmax_bf16.restype = c_int
        lib.snb_causal_softmax_backward.argtypes = [c_void_p, c_void_p, c_void_p, c_uint64, c_uint64, c_uint64,
                                                    c_uint64, c_void_p]
        lib.snb_causal_softmax_backward.restype = c_int
        lib.snb_last_error.argtypes = []
        lib.snb_last_error.restype = c_char_p
        lib.snb_last_path.argtypes = []
        lib.snb_last_path.restype = c_int
        lib.snb_device_status.argtypes = []
        lib.snb_device_status.restype = c_int
        lib.snb_causal_attention_forward.argtypes = [c_void_p, c_void_p, c_void_p, c_void_p, c_uint64, c_uint64,
                                                     c_uint64, c_uint64, c_float, c_uint64, c_void_p, c_int32,
                                                     c_void_p]
        lib.snb_causal_attention_forward.restype = c_int
        lib.snb_causal_attention_backward.argtypes = [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int32,
                                                      c_void_p, c_void_p, c_uint64, c_uint64, c_uint64, c_uint64,
                                                      c_float, c_uint64, c_void_p, c_void_p, c_void_p]
        lib.snb_causal_attention_backward.restype = c_int
        lib.snb_causal_attention_backward_noalloc.argtypes = lib.snb_causal_attention_backward.argtypes
        lib.snb_causal_attention_backward_noalloc.restype = c_int
        lib.snb_cross_entropy.argtypes = [c_void_p, c_void_p, c_uint64, c_uint64, c_void_p, c_uint64,
                                          POINTER(CrossEntropyHead), c_void_p, c_uint64, c_void_p]
        lib.snb_cross_entropy.restype = c_int
        lib.snb_head_cross_entropy.argtypes = [c_void_p, POINTER(GemmArgs), c_void_p, c_uint64, c_uint64, c_uint64,
                                               c_void_p, c_void_p, c_void_p, c_int32]
        lib.snb_head_cross_entropy.restype = c_int
        lib.snb_codebook_cross_entropy.argtypes = [c_void_p, c_void_p, c_int32, c_uint64, c_uint64, c_uint64,
                                                   c_void_p, c_uint64, c_void_p, c_void_p, c_void_p, c_int32]
        lib.snb_codebook_cross_entropy.restype = c_int
        lib.snb_split_heads.argtypes = [c_void_p, c_void_p, c_uint64, c_void_p, c_uint64, POINTER(HeadLayout)]
        lib.snb_split_heads.restype = c_int
        lib.snb_merge_heads.argtypes = [c_void_p, c_void_p, c_uint64, c_void_p, c_uint64, POINTER(HeadLayout)]
        lib.snb_merge_heads.restype = c_int
        lib.snb_permute_heads.argtypes = [c_void_p, c_int32, c_void_p, c_int32, c_uint64, c_void_p, c_int32, c_uint64,
                                          POINTER(HeadLayout)]
        lib.snb_permute_heads.restype = c_int
        lib.snb_rms_norm_forward.argtypes = [c_void_p, c_void_p, c_uint64, c_uint64, c_void_p, c_uint64, c_void_p,
                                             c_void_p, c_uint64, c_float]
        lib.snb_rms_norm_backward.argtypes = [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                              c_uint64, c_uint64, c_uint64]
        lib.snb_rms_norm_stats.argtypes = [c_void_p, c_void_p, c_int32, c_uint64, c_uint64, c_float, c_void_p,
                                           c_void_p, c_void_p, c_int32]
        lib.snb_scale_rows.argtypes = [c_void_p, c_void_p, c_void_p, c_int32, c_void_p, c_int32, c_uint64, c_uint64]
        lib.snb_adamw_step.argtypes = [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_uint64,
                                       POINTER(AdamWHyper)]
        lib.snb_sum_of_squares.argtypes = [c_void_p, c_void_p, c_uint64, c_void_p]
        lib.snb_adamw_step_multi.argtypes = [c_void_p, POINTER(AdamWTensor), c_uint64, POINTER(AdamWHyper), c_float,
                                             c_void_p]
        lib.snb_random_normal.argtypes = [c_void_p, c_void_p, c_int32, c_uint64, c_uint64, c_uint64, c_float]
        lib.snb_random_below.argtypes = [c_void_p, c_void_p, c_uint64, c_uint64, c_uint64, c_uint64]
        for name in ("snb_rms_norm_forward", "snb_rms_norm_backward", "snb_rms_norm_stats", "snb_scale_rows",
                     "snb_adamw_step", "snb_sum_of_squares", "snb_adamw_step_multi", "snb_random_normal",
                     "snb_random_below"):
            getattr(lib, name).restype = c_int
        lib.snb_selftest_bounded_wait.argtypes = [c_void_p, c_uint64]
        lib.snb_selftest_bounded_wait.restype = c_int
        lib.snb_abi_version.argtypes = []
        lib.snb_abi_version.restype = c_int
        _lib = lib
        return lib


def last_error() -> str:
    msg = load().snb_last_error()
    return msg.decode() if msg else ""


def last_path() -> int:
    return load().snb_last_path()


_ = (c_uint16,)  # bf16 buffers travel as raw 16-bit words
