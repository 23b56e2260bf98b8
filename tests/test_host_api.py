"""Host-side logic that needs no GPU: the ABI structures' layout (byte-identical to the reference's repr(C)
`Product`), the MatmulSpec builders (mirroring the unit tests in crates/staleynet-cuda/src/ops/matmul.rs:173-225),
and the shared library: it loads, exports every entry point include/snb_matmul.h declares, and rejects bad
arguments before touching a device."""
import ctypes
import re
from pathlib import Path

import pytest

from staleynet_b200 import _ffi
from staleynet_b200.matmul import BatchStrides, MatmulKernel, MatmulSpec, Storage, WriteMode

ROOT = Path(__file__).resolve().parents[1]


def test_product_layout_matches_the_reference_repr_c():
    # Product { rows, cols, inner: usize, left, right: Operand(3 x usize), output_batch_stride: usize,
    #           scale: f32, accumulate: u32 }  (kernels/matmul.rs:108-157)
    assert ctypes.sizeof(_ffi.Product) == 88
    offsets = {name: getattr(_ffi.Product, name).offset for name, _ in _ffi.Product._fields_}
    assert offsets == {"rows": 0, "cols": 8, "inner": 16, "left": 24, "right": 48, "output_batch_stride": 72,
                       "scale": 80, "accumulate": 84}


def test_new_is_unbatched_row_major_overwrite_with_unit_scale():
    spec = MatmulSpec.new(2, 3, 4)
    assert (spec.rows, spec.cols, spec.inner) == (2, 3, 4)
    assert spec.left is Storage.ROW_MAJOR and spec.right is Storage.ROW_MAJOR
    assert spec.batch == BatchStrides.SINGLE
    assert spec.scale == 1.0 and spec.write is WriteMode.OVERWRITE


def test_builders_set_the_expected_fields():
    spec = (MatmulSpec.new(2, 3, 4).left_transposed().right_transposed().accumulate().scaled(0.25)
            .batched(BatchStrides(count=3, left=8, right=12, output=6)))
    assert spec.left is Storage.TRANSPOSED and spec.right is Storage.TRANSPOSED
    assert spec.write is WriteMode.ACCUMULATE and spec.scale == 0.25
    assert spec.batch == BatchStrides(3, 8, 12, 6)


def test_required_len_accounts_for_the_batch_stride():
    spec = MatmulSpec.new(2, 3, 4).batched(BatchStrides(count=3, left=8, right=0, output=6))
    assert spec.required_len(8, 8) == 24
    assert spec.required_len(0, 8) == 8
    assert spec.required_len(6, 6) == 18


def test_storage_strides_swap_for_a_transpose():
    p = MatmulSpec.new(5, 7, 3).left_transposed().product()
    assert (p.left.row_stride, p.left.col_stride) == (1, 5)
    assert (p.right.row_stride, p.right.col_stride) == (7, 1)
    assert WriteMode.OVERWRITE.flag() == 0 and WriteMode.ACCUMULATE.flag() == 1


def test_kernel_tolerances_follow_the_reference():
    assert MatmulKernel.BLOCKED.tolerance() == 1e-5
    assert MatmulKernel.TENSOR_CORE.tolerance() == 2e-3
    assert MatmulKernel.BF16_TENSOR_CORE.tolerance() == 1e-2


def header_functions():
    text = (ROOT / "include" / "snb_matmul.h").read_text()
    return sorted(set(re.findall(r"SNB_API\s+[\w\s\*]*?\b(snb_\w+)\s*\(", text)))


def test_library_loads_and_exports_every_declared_symbol():
    lib = _ffi.load()
    declared = header_functions()
    assert declared, "no declarations found in include/snb_matmul.h"
    for name in declared:
        assert hasattr(lib, name), f"{name} declared in the header but not exported"
    assert sorted(_ffi.EXPORTED_SYMBOLS) == declared
    assert lib.snb_abi_version() == 106


def call_matmul(rows, cols, inner, left_len, right_len, output_len, count=1, precision=_ffi.PRECISION_F32):
    lib = _ffi.load()
    p = MatmulSpec.new(rows, cols, inner).product()
    fake = 0x1000  # never dereferenced: every case below fails validation or has nothing to compute
    return lib.snb_matmul(None, ctypes.byref(p), count, fake, left_len, fake, right_len, fake, output_len, precision)


def test_undersized_operands_are_rejected_in_the_reference_order():
    assert call_matmul(4, 5, 6, 23, 30, 20) == _ffi.ERR_LEFT_TOO_SMALL
    assert "left operand too small" in _ffi.last_error()
    assert call_matmul(4, 5, 6, 24, 29, 20) == _ffi.ERR_RIGHT_TOO_SMALL
    assert call_matmul(4, 5, 6, 24, 30, 19) == _ffi.ERR_OUTPUT_TOO_SMALL
    assert "output too small" in _ffi.last_error()


def test_invalid_arguments_are_reported_not_aborted():
    assert call_matmul(4, 5, 6, 24, 30, 20, count=0) == _ffi.ERR_INVALID_ARGUMENT
    assert call_matmul(4, 5, 6, 24, 30, 20, precision=7) == _ffi.ERR_INVALID_ARGUMENT
    lib = _ffi.load()
    assert lib.snb_gemm(None, None) == _ffi.ERR_INVALID_ARGUMENT
    assert lib.snb_causal_softmax(None, None, 0, 5, 2, 3, 1.0, 0) == _ffi.ERR_INVALID_ARGUMENT


def test_empty_products_compute_nothing():
    assert call_matmul(0, 5, 6, 0, 30, 0) == _ffi.OK
    assert _ffi.last_path() == _ffi.PATH_EMPTY


def test_gemm_rejects_a_bf16_accumulate():
    lib = _ffi.load()
    a = _ffi.GemmArgs()
    a.product = MatmulSpec.new(4, 8, 8).accumulate().product()
    a.count = 1
    a.left_type = a.right_type = a.output_type = _ffi.TYPE_BF16
    a.aux_type = _ffi.TYPE_F32
    a.precision = _ffi.PRECISION_BF16
    a.left = a.right = a.output = 0x1000
    a.left_len, a.right_len, a.output_len = 32, 64, 32
    assert lib.snb_gemm(None, ctypes.byref(a)) == _ffi.ERR_UNSUPPORTED


def test_gemm_rejects_mismatched_precision():
    lib = _ffi.load()
    a = _ffi.GemmArgs()
    a.product = MatmulSpec.new(4, 8, 8).product()
    a.count = 1
    a.left_type = a.right_type = _ffi.TYPE_F32
    a.output_type = a.aux_type = _ffi.TYPE_F32
    a.precision = _ffi.PRECISION_BF16
    assert lib.snb_gemm(None, ctypes.byref(a)) == _ffi.ERR_INVALID_ARGUMENT


def test_attention_backward_rejects_sizes_whose_byte_counts_overflow():
    # count * ceil4(2 * queries) * 4 wraps 64 bits to about 128 KiB for this pair; without overflow checks the no-alloc
    # entry point would accept it as fitting its static scratch. Both entry points must refuse it before any CUDA call
    # (the fake pointers are never dereferenced).
    lib = _ffi.load()
    count, queries, keys = 2 ** 30 + 2 ** 15, 2 ** 31 - 65534, 128
    fake = 0x1000
    for fn in (lib.snb_causal_attention_backward_noalloc, lib.snb_causal_attention_backward):
        code = fn(None, fake, fake, fake, fake, _ffi.TYPE_F32, fake, fake, count, queries, keys, 64, 0.125, 0, fake,
                  fake, fake)
        assert code == _ffi.ERR_INVALID_ARGUMENT
        assert "overflow" in _ffi.last_error()


def test_deterministic_switch_is_per_thread_and_returns_the_previous_setting():
    import threading

    lib = _ffi.load()
    assert lib.snb_set_deterministic(1) == 0
    seen = []
    t = threading.Thread(target=lambda: seen.append(lib.snb_set_deterministic(0)))
    t.start()
    t.join()
    assert seen == [0]   # another thread starts from the default
    assert lib.snb_set_deterministic(0) == 1


def test_gemm_rejects_unknown_flags():
    lib = _ffi.load()
    a = _ffi.GemmArgs()
    a.product = MatmulSpec.new(4, 8, 8).product()
    a.count = 1
    a.left_type = a.right_type = a.output_type = a.aux_type = _ffi.TYPE_F32
    a.precision = _ffi.PRECISION_F32
    a.flags = 2
    assert lib.snb_gemm(None, ctypes.byref(a)) == _ffi.ERR_INVALID_ARGUMENT
    assert "flags" in _ffi.last_error()


def test_head_layout_matches_the_reference_struct_and_builders():
    # HeadLayout (kernels/attention.rs:19-69) and its unit tests (ops/attention.rs:104-140).
    from staleynet_b200._ffi import HeadLayout

    assert ctypes.sizeof(HeadLayout) == 64
    L = HeadLayout.dense(2, 5, 4, 8, 32, 16)
    assert (L.batch, L.time, L.heads, L.head_dim, L.width, L.column_offset) == (2, 5, 4, 8, 32, 16)
    assert (L.time_capacity, L.time_offset) == (5, 0)
    c = L.in_cache(9, 3)
    assert (c.time, c.time_capacity, c.time_offset, c.heads, c.head_dim) == (5, 9, 3, 4, 8)


def test_head_permutes_check_the_layout_in_the_reference_order():
    # check_layout (ops/attention.rs:11-18): capacity, then the packed tensor, then the head-major tensor; the
    # messages are the reference's. Fake pointers: every case fails before any device access.
    from staleynet_b200._ffi import HeadLayout

    lib = _ffi.load()
    fake = 0x1000
    L = HeadLayout.dense(2, 5, 3, 4, 38, 13).in_cache(9, 2)
    packed, heads = 2 * 5 * 38, 2 * 3 * 9 * 4
    bad_cap = HeadLayout.dense(2, 5, 3, 4, 38, 13).in_cache(6, 2)
    cases = [(bad_cap, packed, heads, "time range exceeds capacity"),
             (L, packed - 1, heads - 1, "packed tensor too small"),
             (L, packed, heads - 1, "head-major tensor too small")]
    for layout, p_len, h_len, msg in cases:
        assert lib.snb_split_heads(None, fake, p_len, fake, h_len, ctypes.byref(layout)) == _ffi.ERR_INVALID_ARGUMENT
        assert _ffi.last_error() == "HeadLayout: " + msg
        assert lib.snb_merge_heads(None, fake, h_len, fake, p_len, ctypes.byref(layout)) == _ffi.ERR_INVALID_ARGUMENT
        assert _ffi.last_error() == "HeadLayout: " + msg
    assert lib.snb_permute_heads(None, 7, fake, 0, packed, fake, 0, heads, ctypes.byref(L)) == \
        _ffi.ERR_INVALID_ARGUMENT


def test_gemm_head_layouts_must_describe_their_operand():
    from staleynet_b200._ffi import HeadLayout

    lib = _ffi.load()
    B, S, H, d = 2, 128, 2, 64
    w, T = H * d, B * S
    a = _ffi.GemmArgs()
    a.product = MatmulSpec.new(T, w, w).product()
    a.count = 1
    a.left_type = a.right_type = a.output_type = _ffi.TYPE_BF16
    a.aux_type = _ffi.TYPE_F32
    a.precision = _ffi.PRECISION_BF16
    a.left = a.right = a.output = 0x1000
    a.left_len, a.right_len, a.output_len = T * w, w * w, T * w
    wrong = HeadLayout.dense(B, S, H, d, 3 * w, 0)       # width of a fused QKV row: not this operand
    a.left_heads = ctypes.pointer(wrong)
    assert lib.snb_gemm(None, ctypes.byref(a)) == _ffi.ERR_INVALID_ARGUMENT
    assert "left_heads" in _ffi.last_error()
    a.left_heads = None
    a.output_heads = ctypes.pointer(HeadLayout.dense(B, S + 1, H, d, w, 0))   # rows != batch * time
    assert lib.snb_gemm(None, ctypes.byref(a)) == _ffi.ERR_INVALID_ARGUMENT
    assert "output_heads" in _ffi.last_error()
    big = HeadLayout.dense(B, S, H, d, w, 0).in_cache(2 * S, 0)   # the head-major output holds more than T * w
    a.output_heads = ctypes.pointer(big)
    assert lib.snb_gemm(None, ctypes.byref(a)) == _ffi.ERR_OUTPUT_TOO_SMALL


def test_sm_budget_is_per_thread_and_returns_the_previous_setting():
    import threading

    lib = _ffi.load()
    assert lib.snb_set_sm_budget(100) == 0
    seen = []
    t = threading.Thread(target=lambda: seen.append(lib.snb_set_sm_budget(0)))
    t.start()
    t.join()
    assert seen == [0]
    assert lib.snb_set_sm_budget(-5) == 100      # non-positive: no cap
    assert lib.snb_set_sm_budget(0) == 0
