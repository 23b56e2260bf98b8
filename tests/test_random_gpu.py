"""GPU parity of the device generator (snb_random_normal / snb_random_below) with the reference's `Random`
(crates/staleynet-model/src/random.rs:27-70) as restated by the oracle, which the CPU suite pins to the published
SplitMix64 sequence (tests/test_oracle.py). Integer draws must be identical; normal values may differ from the host
libm's logf / cosf in an f32's last bits, so they are bounded in ulps and counted for exact agreement."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import oracle as o  # noqa: E402
from staleynet_b200.matmul import DeviceRandom, Gpu, SnbError  # noqa: E402

pytestmark = pytest.mark.gpu

GAMMA = 0x9E3779B97F4A7C15
MASK = (1 << 64) - 1


@pytest.fixture(scope="module")
def gpu():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return Gpu(0)


def host_after(seed: int, draws: int) -> o.Random:
    """The oracle generator in the state Random::new(seed) reaches after `draws` draws."""
    return o.Random((seed + draws * GAMMA) & MASK)


def ulps(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    ia = a.view(np.int32).astype(np.int64)
    ib = b.view(np.int32).astype(np.int64)
    ia = np.where(ia < 0, -(ia & 0x7FFFFFFF), ia)
    ib = np.where(ib < 0, -(ib & 0x7FFFFFFF), ib)
    return np.abs(ia - ib)


@pytest.mark.parametrize("seed,std", [(0, 1.0), (12345, 0.0361)])
def test_normal_fill_matches_the_reference_stream(gpu, seed, std):
    n = 6000
    out = torch.empty(n, device="cuda", dtype=torch.float32)
    assert gpu.random_normal(out, seed, 0, std) == 2 * n
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    want = o.Random(seed).normals(n, std)
    d = ulps(got, want)
    assert d.max() <= 8, d.max()
    assert np.mean(d == 0) > 0.5, np.mean(d == 0)
    gpu.device_status()


def test_consecutive_fills_continue_the_stream_and_bf16_rounds_the_f32_value(gpu):
    rng = DeviceRandom(gpu, 0)
    a = rng.normal_(torch.empty(1000, device="cuda", dtype=torch.float32))
    b = rng.normal_(torch.empty(777, device="cuda", dtype=torch.float32), 0.5)
    assert rng.draws == 2 * 1777
    host = o.Random(0)
    want_a, want_b = host.normals(1000), host.normals(777, 0.5)
    torch.cuda.synchronize()
    assert ulps(a.cpu().numpy(), want_a).max() <= 8
    assert ulps(b.cpu().numpy(), want_b).max() <= 8
    # bf16 output = the same value rounded to nearest even
    bf = torch.empty(1000, device="cuda", dtype=torch.bfloat16)
    gpu.random_normal(bf, 0, 0, 1.0)
    torch.cuda.synchronize()
    assert torch.equal(bf.cpu(), a.cpu().to(torch.bfloat16))


def test_skipping_draws_lands_on_the_same_values(gpu):
    # 3M values: several grid-stride rounds; checked at sampled positions against a host generator moved there.
    n, first = 3_000_000, 41
    out = torch.empty(n, device="cuda", dtype=torch.float32)
    gpu.random_normal(out, 7, first, 1.0)
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    for i in (0, 1, 606_207, 606_208, 2_999_999):
        want = host_after(7, first + 2 * i).normals(1)
        assert ulps(got[i:i + 1], want).max() <= 8, i


def test_below_fill_is_identical(gpu):
    n = 5000
    out = torch.empty(n, device="cuda", dtype=torch.int32)
    assert gpu.random_below(out, 1024, 0, 3) == 3 + n
    torch.cuda.synchronize()
    want = host_after(0, 3).belows(n, 1024)
    assert np.array_equal(out.cpu().numpy().astype(np.uint32), want)


def test_invalid_arguments_raise(gpu):
    with pytest.raises(SnbError):
        gpu.random_below(torch.empty(4, device="cuda", dtype=torch.int32), 0, 0)
    with pytest.raises(SnbError):
        gpu.random_normal(torch.empty(4, device="cuda", dtype=torch.float16), 0)
