"""snb_causal_attention_backward_noalloc: the fused attention backward with its row-statistics scratch in a static
__device__ array instead of a stream-ordered allocation. Two calls in a row on different inputs must give what the
allocating entry point gives (dK and dV bit for bit; dQ, summed by unordered TMA reductions, to f32 rounding), and a
call whose scratch would not fit must be refused before any buffer is touched. This file sorts last so that it also
runs after every other GPU test in the same process."""
import pytest

torch = pytest.importorskip("torch")

from staleynet_b200 import _ffi  # noqa: E402
from staleynet_b200.matmul import Gpu  # noqa: E402

pytestmark = pytest.mark.gpu


def _inputs(seed, count, sq, sk):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    mk = lambda n: torch.randn(count, n, 64, device="cuda", generator=g).bfloat16()  # noqa: E731
    return mk(sq), mk(sk), mk(sk), mk(sq)


def test_no_alloc_backward_matches_the_allocating_entry_point_on_two_calls_in_a_row():
    gpu = Gpu(0)
    scale = 0.125
    for seed, (count, sq, sk, offset) in enumerate([(3, 384, 384, 0), (2, 300, 520, 220)]):
        q, k, v, do = _inputs(seed, count, sq, sk)
        out = torch.empty(count, sq, 64, device="cuda")
        lse = torch.empty(count, sq, device="cuda")
        gpu.causal_attention_forward(q, k, v, out, scale, offset, lse)
        ref = [torch.empty(count, n, 64, device="cuda") for n in (sq, sk, sk)]
        got = [torch.full((count, n, 64), 9.0, device="cuda") for n in (sq, sk, sk)]
        gpu.causal_attention_backward(q, k, v, out, do, lse, *ref, scale, offset)
        gpu.causal_attention_backward(q, k, v, out, do, lse, *got, scale, offset, no_alloc=True)
        torch.cuda.synchronize()
        assert _ffi.load().snb_device_status() == _ffi.OK
        assert torch.equal(got[1], ref[1]) and torch.equal(got[2], ref[2]), "dk/dv"
        err = (torch.linalg.vector_norm(got[0] - ref[0]) / torch.linalg.vector_norm(ref[0])).item()
        assert err < 1e-5, "dq"


def test_no_alloc_backward_refuses_what_its_scratch_cannot_hold():
    gpu = Gpu(0)
    # 2048 matrices x 1024 queries need 16 MiB of row statistics; the static scratch holds 8 MiB. Small tensors are
    # enough: the size check comes before any buffer is read or written.
    q, k, v, do = _inputs(0, 1, 128, 128)
    out = torch.empty(1, 128, 64, device="cuda")
    lse = torch.empty(1, 128, device="cuda")
    dq, dk, dv = (torch.empty(1, 128, 64, device="cuda") for _ in range(3))
    lib = gpu.lib
    h = gpu._stream_handle()
    code = lib.snb_causal_attention_backward_noalloc(h, q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(),
                                                     _ffi.TYPE_F32, do.data_ptr(), lse.data_ptr(), 2048, 1024, 1024,
                                                     64, 0.125, 0, dq.data_ptr(), dk.data_ptr(), dv.data_ptr())
    assert code == _ffi.ERR_INVALID_ARGUMENT
    assert b"static scratch" in lib.snb_last_error()
    torch.cuda.synchronize()
    assert _ffi.load().snb_device_status() == _ffi.OK
