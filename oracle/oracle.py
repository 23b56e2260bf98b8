"""TEST INFRASTRUCTURE ONLY: ctypes access to the CPU oracle (oracle/snb_oracle.c).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use this module, as the checker or as the
reported CPU baseline; the product library never loads it. The C file restates the reference's arithmetic
(crates/staleynet-cuda/src/reference.rs and crates/staleynet-model/src/random.rs; citations in the C source).
"""
from __future__ import annotations

import ctypes
import os
import shutil
import subprocess
import threading
from ctypes import POINTER, c_double, c_float, c_int, c_uint16, c_uint32, c_uint64, c_void_p
from pathlib import Path

import numpy as np

ORACLE_DIR = Path(__file__).resolve().parent
SOURCE = ORACLE_DIR / "snb_oracle.c"
BUILD_DIR = ORACLE_DIR / "_build"
LIB_PATH = BUILD_DIR / "libsnb_oracle.so"


class Operand(ctypes.Structure):
    _fields_ = [("row_stride", c_uint64), ("col_stride", c_uint64), ("batch_stride", c_uint64)]


class Product(ctypes.Structure):
    _fields_ = [("rows", c_uint64), ("cols", c_uint64), ("inner", c_uint64), ("left", Operand), ("right", Operand),
                ("output_batch_stride", c_uint64), ("scale", c_float), ("accumulate", c_uint32)]


def build(force: bool = False) -> Path:
    """Compiles the oracle with gcc (OpenMP for the all-cores baseline). No FMA contraction: -O2 on baseline
    x86-64 keeps every `sum += a*b` a separate multiply and add, like the reference's Rust loop."""
    header = ORACLE_DIR.parent / "include" / "snb_matmul.h"
    newest = max(SOURCE.stat().st_mtime, header.stat().st_mtime, Path(__file__).stat().st_mtime)
    if not force and LIB_PATH.exists() and LIB_PATH.stat().st_mtime >= newest:
        return LIB_PATH
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        raise RuntimeError("gcc not found")
    BUILD_DIR.mkdir(exist_ok=True)
    tmp = LIB_PATH.with_suffix(f".so.{os.getpid()}.tmp")  # concurrent builders (spawned test ranks) never collide
    cmd = [cc, "-O2", "-fPIC", "-shared", "-fopenmp", "-ffp-contract=off", "-o", str(tmp), str(SOURCE), "-lm"]
    subprocess.run(cmd, check=True, capture_output=True, text=True)
    tmp.replace(LIB_PATH)
    return LIB_PATH


_lock = threading.Lock()
_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    with _lock:
        if _lib is None:
            build()
            L = ctypes.CDLL(str(LIB_PATH))
            fp = POINTER(c_float)
            L.snb_oracle_matmul.argtypes = [POINTER(Product), c_uint64, fp, fp, fp]
            L.snb_oracle_matmul_rows.argtypes = [POINTER(Product), c_uint64, fp, fp, fp, c_uint64, c_uint64]
            L.snb_oracle_matmul_parallel.argtypes = [POINTER(Product), c_uint64, fp, fp, fp, c_uint64, c_uint64, c_int]
            L.snb_oracle_matmul_parallel.restype = c_int
            L.snb_oracle_matmul_f64.argtypes = [POINTER(Product), c_uint64, fp, fp, POINTER(c_double)]
            L.snb_oracle_round_tf32.argtypes = [fp, fp, c_uint64]
            L.snb_oracle_round_bf16.argtypes = [fp, fp, POINTER(c_uint16), c_uint64]
            L.snb_oracle_next_u64.argtypes = [POINTER(c_uint64)]
            L.snb_oracle_next_u64.restype = c_uint64
            L.snb_oracle_uniform.argtypes = [POINTER(c_uint64)]
            L.snb_oracle_uniform.restype = c_float
            L.snb_oracle_below.argtypes = [POINTER(c_uint64), c_uint64]
            L.snb_oracle_below.restype = c_uint64
            L.snb_oracle_normal.argtypes = [POINTER(c_uint64)]
            L.snb_oracle_normal.restype = c_float
            L.snb_oracle_fill_normal.argtypes = [POINTER(c_uint64), c_float, fp, c_uint64]
            L.snb_oracle_fill_below.argtypes = [POINTER(c_uint64), c_uint64, POINTER(c_uint32), c_uint64]
            L.snb_oracle_fill_lcg.argtypes = [c_uint64, fp, c_uint64]
            L.snb_oracle_gelu.argtypes = [c_float]
            L.snb_oracle_gelu.restype = c_float
            L.snb_oracle_gelu_derivative.argtypes = [c_float]
            L.snb_oracle_gelu_derivative.restype = c_float
            L.snb_oracle_gelu_fill.argtypes = [fp, fp, c_uint64]
            L.snb_oracle_gelu_derivative_fill.argtypes = [fp, fp, c_uint64]
            L.snb_oracle_causal_softmax.argtypes = [fp, c_uint64, c_uint64, c_uint64, c_float, c_uint64]
            L.snb_oracle_softmax_backward.argtypes = [fp, fp, c_uint64, c_uint64]
            L.snb_oracle_cross_entropy.argtypes = [fp, POINTER(c_uint32), c_uint64, c_uint64, c_uint64, c_uint64,
                                                   c_uint64, c_uint64, c_float, fp, fp]
            L.snb_oracle_rms_norm_forward.argtypes = [fp, fp, c_uint64, c_uint64, c_float, fp, fp]
            L.snb_oracle_rms_norm_backward.argtypes = [fp, fp, fp, fp, c_uint64, c_uint64, fp, fp]
            L.snb_oracle_adamw_step.argtypes = [fp, fp, fp, fp, c_uint64, c_float, c_float, c_float, c_float, c_float,
                                                c_uint32]
            L.snb_oracle_sum_of_squares.argtypes = [fp, c_uint64]
            L.snb_oracle_sum_of_squares.restype = c_double
            L.snb_oracle_max_threads.restype = c_int
            _lib = L
    return _lib


def _f(a: np.ndarray):
    assert a.dtype == np.float32 and a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(POINTER(c_float))


def product(rows, cols, inner, left_strides, right_strides, output_batch_stride, scale=1.0, accumulate=False):
    """A Product from (row_stride, col_stride, batch_stride) triples."""
    return Product(rows, cols, inner, Operand(*left_strides), Operand(*right_strides), output_batch_stride, scale,
                   1 if accumulate else 0)


def storage_strides(transposed: bool, rows: int, cols: int, batch_stride: int):
    """`Storage::operand` (ops/matmul.rs:24-33)."""
    return (1, rows, batch_stride) if transposed else (cols, 1, batch_stride)


def matmul(p: Product, count: int, left: np.ndarray, right: np.ndarray, output: np.ndarray) -> None:
    """reference::matmul (reference.rs:18-38), in place on `output`."""
    lib().snb_oracle_matmul(ctypes.byref(p), count, _f(left), _f(right), _f(output))


def matmul_rows(p: Product, count: int, left, right, output, row_begin: int, row_end: int, threads: int = 0) -> int:
    """The reference loop over output rows [row_begin, row_end) on `threads` OpenMP threads (0 = all)."""
    return lib().snb_oracle_matmul_parallel(ctypes.byref(p), count, _f(left), _f(right), _f(output), row_begin,
                                            row_end, threads)


def matmul_f64(p: Product, count: int, left, right, output: np.ndarray) -> None:
    assert output.dtype == np.float64
    lib().snb_oracle_matmul_f64(ctypes.byref(p), count, _f(left), _f(right),
                                output.ctypes.data_as(POINTER(c_double)))


def round_tf32(a: np.ndarray) -> np.ndarray:
    a = np.ascontiguousarray(a, dtype=np.float32)
    out = np.empty_like(a)
    lib().snb_oracle_round_tf32(_f(a), _f(out), a.size)
    return out


def round_bf16(a: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """Returns (values rounded to bf16 as f32, raw bf16 bits as uint16)."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    out = np.empty_like(a)
    bits = np.empty(a.shape, dtype=np.uint16)
    lib().snb_oracle_round_bf16(_f(a), _f(out), bits.ctypes.data_as(POINTER(c_uint16)), a.size)
    return out, bits


class Random:
    """`Random` (crates/staleynet-model/src/random.rs:27-70) over the C restatement."""

    def __init__(self, seed: int):
        self.state = c_uint64(seed)

    def next_u64(self) -> int:
        return lib().snb_oracle_next_u64(ctypes.byref(self.state))

    def uniform(self) -> float:
        return lib().snb_oracle_uniform(ctypes.byref(self.state))

    def below(self, bound: int) -> int:
        return lib().snb_oracle_below(ctypes.byref(self.state), bound)

    def normal(self) -> float:
        return lib().snb_oracle_normal(ctypes.byref(self.state))

    def normals(self, n: int, std: float = 1.0) -> np.ndarray:
        out = np.empty(n, dtype=np.float32)
        lib().snb_oracle_fill_normal(ctypes.byref(self.state), std, _f(out), n)
        return out

    def belows(self, n: int, bound: int) -> np.ndarray:
        out = np.empty(n, dtype=np.uint32)
        lib().snb_oracle_fill_below(ctypes.byref(self.state), bound, out.ctypes.data_as(POINTER(c_uint32)), n)
        return out


def lcg_values(count: int, seed: int) -> np.ndarray:
    """The parity tests' LCG inputs in roughly [-1, 1] (kernels_match_reference.rs:26-38)."""
    out = np.empty(count, dtype=np.float32)
    lib().snb_oracle_fill_lcg(seed, _f(out), count)
    return out


def head_indices(layout) -> tuple[np.ndarray, np.ndarray]:
    """(packed index, head-major index) of every element a head permute moves, enumerated as `HeadLayout::element`
    does (dim fastest, then step, head, batch) with `packed_index` / `head_major_index`
    (crates/staleynet-cuda/src/kernels/attention.rs:71-96). `layout` has the eight HeadLayout fields."""
    L = layout
    e = np.arange(L.batch * L.heads * L.time * L.head_dim, dtype=np.int64)
    dim = e % L.head_dim
    step = (e // L.head_dim) % L.time
    head = (e // (L.head_dim * L.time)) % L.heads
    batch = e // (L.head_dim * L.time * L.heads)
    packed = (batch * L.time + step) * L.width + L.column_offset + head * L.head_dim + dim
    head_major = ((batch * L.heads + head) * L.time_capacity + L.time_offset + step) * L.head_dim + dim
    return packed, head_major


def split_heads(packed: np.ndarray, head_major: np.ndarray, layout) -> None:
    """`split_heads` (kernels/attention.rs:112-121): head_major[head_major_index] = packed[packed_index]."""
    p, h = head_indices(layout)
    head_major[h] = packed[p]


def merge_heads(head_major: np.ndarray, packed: np.ndarray, layout) -> None:
    """`merge_heads` (kernels/attention.rs:129-138): packed[packed_index] = head_major[head_major_index]; other
    columns untouched."""
    p, h = head_indices(layout)
    packed[p] = head_major[h]


def gelu(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty_like(x)
    lib().snb_oracle_gelu_fill(_f(x), _f(out), x.size)
    return out


def gelu_derivative(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty_like(x)
    lib().snb_oracle_gelu_derivative_fill(_f(x), _f(out), x.size)
    return out


def causal_softmax(scores: np.ndarray, queries: int, keys: int, scale: float, query_offset: int) -> None:
    """reference::causal_softmax (reference.rs:100-120), in place."""
    rows = scores.size // keys
    lib().snb_oracle_causal_softmax(_f(scores), rows, queries, keys, scale, query_offset)


def softmax_backward(probabilities: np.ndarray, grad: np.ndarray, cols: int) -> None:
    """reference::softmax_backward (reference.rs:122-137), in place on grad."""
    lib().snb_oracle_softmax_backward(_f(probabilities), _f(grad), grad.size // cols, cols)


def cross_entropy(logits: np.ndarray, targets: np.ndarray, cols: int, column_offset: int, classes: int,
                  target_stride: int, target_offset: int, grad_scale: float, losses: np.ndarray,
                  logits_grad: np.ndarray) -> None:
    """reference::cross_entropy (reference.rs:139-166) for one head, in place on losses and logits_grad."""
    targets = np.ascontiguousarray(targets, dtype=np.uint32)
    rows = losses.size
    lib().snb_oracle_cross_entropy(_f(logits), targets.ctypes.data_as(POINTER(c_uint32)), rows, cols, column_offset,
                                   classes, target_stride, target_offset, grad_scale, _f(losses), _f(logits_grad))


def rms_norm_forward(x: np.ndarray, gain: np.ndarray, cols: int, epsilon: float):
    """reference::rms_norm_forward (reference.rs:60-77): returns (output, inv_rms)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    gain = np.ascontiguousarray(gain, dtype=np.float32)
    rows = x.size // cols
    out = np.empty_like(x)
    inv = np.empty(rows, np.float32)
    lib().snb_oracle_rms_norm_forward(_f(x), _f(gain), rows, cols, epsilon, _f(out), _f(inv))
    return out, inv


def rms_norm_backward(dy: np.ndarray, x: np.ndarray, gain: np.ndarray, inv_rms: np.ndarray, cols: int):
    """reference::rms_norm_backward (reference.rs:79-98): returns (input_grad, gain_grad)."""
    dy, x = (np.ascontiguousarray(a, dtype=np.float32) for a in (dy, x))
    gain, inv_rms = (np.ascontiguousarray(a, dtype=np.float32) for a in (gain, inv_rms))
    dx = np.empty_like(x)
    dg = np.zeros(cols, np.float32)
    lib().snb_oracle_rms_norm_backward(_f(dy), _f(x), _f(gain), _f(inv_rms), x.size // cols, cols, _f(dx), _f(dg))
    return dx, dg


def adamw_step(parameter, gradient, first, second, learning_rate, beta1, beta2, epsilon, weight_decay, step) -> None:
    """The reference's AdamW update (kernels/optimizer.rs:47-71), in place on parameter and the moments."""
    lib().snb_oracle_adamw_step(_f(parameter), _f(np.ascontiguousarray(gradient, dtype=np.float32)), _f(first),
                                _f(second), parameter.size, learning_rate, beta1, beta2, epsilon, weight_decay, step)


def sum_of_squares(values: np.ndarray) -> float:
    return lib().snb_oracle_sum_of_squares(_f(np.ascontiguousarray(values, dtype=np.float32)), values.size)


def max_threads() -> int:
    return lib().snb_oracle_max_threads()


def relative_error(expected: np.ndarray, actual: np.ndarray) -> float:
    """max|delta| / max|expected| (kernels_match_reference.rs:41-52)."""
    expected = np.asarray(expected, dtype=np.float64).ravel()
    actual = np.asarray(actual, dtype=np.float64).ravel()
    magnitude = max(float(np.finfo(np.float32).eps), float(np.max(np.abs(expected))) if expected.size else 0.0)
    worst = float(np.max(np.abs(expected - actual))) if expected.size else 0.0
    return worst / magnitude


def relative_frobenius(expected: np.ndarray, actual: np.ndarray) -> float:
    """||actual - expected||_F / ||expected||_F, the north star's tolerance metric."""
    expected = np.asarray(expected, dtype=np.float64).ravel()
    actual = np.asarray(actual, dtype=np.float64).ravel()
    denom = float(np.linalg.norm(expected))
    return float(np.linalg.norm(actual - expected)) / (denom if denom > 0 else 1.0)


_ = c_void_p
