"""The reference's other callers of `Gpu::matmul`, at their own shapes, through the C ABI against the oracle: the
vocoder's inverse STFT (crates/staleynet-model/src/vocoder/istft.rs:105-133) and multi-resolution spectral loss
(vocoder/loss.rs:205-244; resolutions loss.rs:37-39), the data crate's mel features (staleynet-data/src/
features.rs:78-89) and the tokenizer's nearest-centroid search (tokenizer.rs:158). Their bin counts (fft/2 + 1 =
257, 513, 1025) give operand strides that are no multiple of 16 bytes, so these products take the strided SIMT
kernel rather than TMA; they must still match the reference within its kernel tolerances (1e-5 f32, 2e-3 tf32)."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import oracle as o  # noqa: E402
from staleynet_b200 import _ffi  # noqa: E402
from staleynet_b200.matmul import Gpu, MatmulKernel, MatmulSpec  # noqa: E402

pytestmark = pytest.mark.gpu

ROWS = 300                   # spectrogram frames / search points per call (any count; the shapes are the point)
MEL_BANDS = 128              # vocoder/config.rs:45
RESOLUTIONS = (512, 1024, 2048)


@pytest.fixture(scope="module")
def gpu():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return Gpu(0)


def to_oracle(spec):
    p = spec.product()
    return o.product(p.rows, p.cols, p.inner, (p.left.row_stride, p.left.col_stride, 0),
                     (p.right.row_stride, p.right.col_stride, 0), 0, p.scale, bool(p.accumulate))


def run(gpu, kernel, chain, seed):
    """`chain`: [(spec, left numel, right numel)] writing one output in turn (later specs may accumulate);
    returns (expected, actual, paths)."""
    gpu.matmul_kernel = kernel
    out_len = chain[0][0].rows * chain[0][0].cols
    expected = np.zeros(out_len, np.float32)
    actual = torch.zeros(out_len, device="cuda")
    paths = []
    for i, (spec, n_left, n_right) in enumerate(chain):
        left = o.lcg_values(n_left, seed + 2 * i)
        right = o.lcg_values(n_right, seed + 2 * i + 1)
        o.matmul_rows(to_oracle(spec), 1, left, right, expected, 0, spec.rows)
        gpu.matmul(spec, torch.from_numpy(left).cuda(), torch.from_numpy(right).cuda(), actual)
        paths.append(_ffi.last_path())
    torch.cuda.synchronize()
    return expected, actual.cpu().numpy(), paths


def caller_chains():
    cases = {}
    for fft in RESOLUTIONS:
        bins = fft // 2 + 1
        fwd = MatmulSpec.new(ROWS, fft, bins)
        cases[f"istft.forward fft{fft}"] = [(fwd, ROWS * bins, bins * fft), (fwd.accumulate(), ROWS * bins, bins * fft)]
        cases[f"istft.backward fft{fft}"] = [(MatmulSpec.new(ROWS, bins, fft).right_transposed(), ROWS * fft, bins * fft)]
        cases[f"loss.analyze fft{fft}"] = [(MatmulSpec.new(ROWS, bins, fft), ROWS * fft, fft * bins)]
        back = MatmulSpec.new(ROWS, fft, bins).right_transposed()
        cases[f"loss.backward frames fft{fft}"] = [(back, ROWS * bins, fft * bins),
                                                   (back.accumulate(), ROWS * bins, fft * bins)]
    bins = 1024 // 2 + 1
    cases["loss.analyze mel"] = [(MatmulSpec.new(ROWS, MEL_BANDS, bins), ROWS * bins, bins * MEL_BANDS)]
    cases["loss.backward mel"] = [(MatmulSpec.new(ROWS, bins, MEL_BANDS).right_transposed(), ROWS * MEL_BANDS,
                                   bins * MEL_BANDS)]
    cases["features.mel"] = [(MatmulSpec.new(ROWS, MEL_BANDS, bins), ROWS * bins, bins * MEL_BANDS)]
    cases["tokenizer.nearest centroid"] = [(MatmulSpec.new(ROWS, 1024, 48).right_transposed(), ROWS * 48, 1024 * 48)]
    return cases


@pytest.mark.parametrize("kernel", [MatmulKernel.BLOCKED, MatmulKernel.TENSOR_CORE])
@pytest.mark.parametrize("name", sorted(caller_chains()))
def test_caller_shapes_match_the_reference(gpu, kernel, name):
    chain = caller_chains()[name]
    expected, actual, paths = run(gpu, kernel, chain, seed=31)
    assert all(p != _ffi.PATH_NONE for p in paths), paths
    assert o.relative_error(expected, actual) < kernel.tolerance(), (name, kernel)
    gpu.device_status()
